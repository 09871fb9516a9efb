// ec_comm.h -- run-time loaded NCCL used by k-means (ec_comm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace ec {

// true after ec_comm_init: one device per process, `world` processes
bool comm_process_mode();
// number of ranks that take part in the k-means exchange
int comm_world();
// rank of local device `local_index` (process mode: this process's rank)
int comm_rank(int local_index);
// create the communicator over the local devices when there are several
int comm_ensure_local();
// EC_ESTATE when the process-mode communicator was aborted
int comm_check_ready();
// clear the shared failure flag before a multi-rank operation
void comm_begin();
// a local rank failed: the others stop waiting on their collectives
void comm_mark_failed();
// host-side meeting of the `nlocal` local ranks before their first
// collective of an operation (bounded): a rank that failed earlier makes the
// others return before they post any NCCL work, so nothing waits on it
int comm_rendezvous(int local_index, int nlocal);
// after a failed multi-rank operation, once every local rank has returned and
// before device memory is freed: abort every communicator and forget them
void comm_abort_all();
// in-place sum all-reduce of `count` floats on `st`; waits (bounded) for it
int comm_allreduce_sum_f32(int local_index, float* buf, size_t count, cudaStream_t st);
// point-to-point and broadcast of `count` floats on `st` (bounded waits)
int comm_send_f32(int local_index, const float* buf, size_t count, int peer, cudaStream_t st);
int comm_recv_f32(int local_index, float* buf, size_t count, int peer, cudaStream_t st);
int comm_bcast_f32(int local_index, float* buf, size_t count, int root, cudaStream_t st);
void comm_destroy();

}  // namespace ec
