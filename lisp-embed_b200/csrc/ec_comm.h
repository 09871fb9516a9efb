// ec_comm.h -- run-time loaded NCCL used by k-means (ec_comm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace ec {

// true after ec_comm_init: one device per process, `world` processes
bool comm_process_mode();
// number of ranks that take part in the k-means all-reduce
int comm_world();
// create the communicator over the local devices when there are several
int comm_ensure_local();
// in-place sum all-reduce of `count` floats on `st`; waits (bounded) for it
int comm_allreduce_sum_f32(int local_index, float* buf, size_t count, cudaStream_t st);
void comm_destroy();

}  // namespace ec
