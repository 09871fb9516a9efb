// ec_state.h -- library-internal state shared by the host translation units:
// the per-device context (stream, uploaded tensors, packed model weights,
// workspace, resident index), error reporting and checked allocation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/embedcuda.h"
#include "ec_kernels.h"

namespace ec {

using bf16 = __nv_bfloat16;

struct Tensor {
  void* p = nullptr;
  int dtype = kDtF32;  // kDtF32 or kDtBf16 on the device (F16 is widened to F32)
  std::vector<int64_t> shape;
  size_t numel = 0;
};

struct BertLayerW {
  bf16 *wqkv = nullptr, *wo = nullptr, *wff = nullptr, *wout = nullptr;
  float *bqkv = nullptr, *bo = nullptr, *ln1g = nullptr, *ln1b = nullptr;
  float *bff = nullptr, *bout = nullptr, *ln2g = nullptr, *ln2b = nullptr;
};

struct LlamaLayerW {
  float *in_ln = nullptr, *post_ln = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  bf16 *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
};

// EmbeddingGemma layer (gemma.lisp:149-212)
struct GemmaLayerW {
  float *in_ln = nullptr, *post_ln = nullptr, *pre_ff_ln = nullptr, *post_ff_ln = nullptr;
  float *q_norm = nullptr, *k_norm = nullptr, *ple_norm = nullptr;
  bf16 *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
  bf16 *wpp = nullptr;        // this layer's rows of the per-layer projection [P, H]
  bf16 *wple_gate = nullptr;  // [P, H]
  bf16 *wple_proj = nullptr;  // [H, P]
  float scalar = 1.f;
  int rope = 0;               // 0: theta 1e4 table, 1: theta 1e6 (full_attention)
};

struct ModelW {
  int family = 0;  // EC_FAMILY_*
  int H = 0, layers = 0, heads = 0, kv_heads = 0, hd = 0, F = 0;
  int out_dim = 0;            // embedding width (H except Gemma's projection)
  int ple_dim = 0;            // Gemma per-layer-input width
  std::vector<GemmaLayerW> gl;
  float *ple_norm = nullptr, *w_out = nullptr;   // Gemma [P], [out_dim, H] fp32
  float *cos2_t = nullptr, *sin2_t = nullptr;    // Gemma theta-1e6 RoPE tables
  int pooling = 0;  // 0 first token, 1 mean, 2 last token
  int pos_offset = 0, vocab = 0, max_pos = 0;
  double eps = 1e-6, theta = 10000.0;
  const void* word = nullptr;
  int word_dt = kDtF32;
  const void* pos = nullptr;
  int pos_dt = kDtF32;
  const void* type0 = nullptr;
  int type_dt = kDtF32;
  float *emb_g = nullptr, *emb_b = nullptr;
  float* relbias = nullptr;  // MPNet [heads][2 * rel_max - 1] * log2(e)
  int rel_max = 0;
  std::vector<BertLayerW> bl;
  std::vector<LlamaLayerW> ll;
  float *final_norm = nullptr, *cos_t = nullptr, *sin_t = nullptr;
  std::vector<void*> owned;
};

struct IndexW {
  int64_t n = 0;
  int d = 0, k = 0;
  float* x = nullptr;          // [n, d]
  float* cent = nullptr;       // [k, d]
  uint32_t* lists = nullptr;   // [n]
  int64_t* offs = nullptr;     // [k + 1]
  std::vector<int64_t> h_offs; // host copy
  std::vector<void*> owned;
  void* sws = nullptr;         // search workspace
  size_t sws_bytes = 0;
  void* cent_b = nullptr;      // bf16 centroids for tensor-core probe scores (lazy, owned)
  float* cent_max = nullptr;   // upper bound of the centroid norms
};

struct ProfAcc {
  double ms = 0, flops = 0, bytes = 0;
  long long launches = 0;
};

struct PendingEv {
  int cls;  // 0 gemm, 1 attention, 2 rows
  double flops, bytes;
  int e0, e1;
};

struct Device {
  int ordinal = 0;
  std::vector<cudaEvent_t> evpool;  // profiling events, reused
  std::vector<PendingEv> pend;      // launches awaiting their elapsed time
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  std::map<std::string, Tensor> uploads;
  ModelW model;
  IndexW index;
  unsigned* status = nullptr;  // device status word of bounded waits
  // forward workspace
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int ws_tokens = 0, ws_seqs = 0;
  // pinned host staging
  void* pin = nullptr;
  size_t pin_bytes = 0;
  size_t allocated = 0;
  // freed blocks kept for an allocation of the same size (dev_alloc /
  // dev_free), oldest first; every use of them is on `stream`, so stream
  // order makes the reuse safe
  std::vector<std::pair<void*, size_t>> free_blocks;
  size_t free_bytes = 0;
  // pinned staging ring of large uploads (upload_h2d)
  static constexpr int kStages = 4;
  void* stage[kStages] = {};
  cudaEvent_t stage_ev[kStages] = {};
  // pinned mirror of the status word (read with the stream's last copy)
  unsigned* status_host = nullptr;
  // pinned landing area of small search results (kResHostBytes)
  static constexpr size_t kResHostBytes = size_t{64} << 10;
  void* res_host = nullptr;
  // captured forwards of small host batches: the whole upload -> forward ->
  // download sequence of one set of sequence lengths as a CUDA graph, valid
  // for the workspace and staging it was captured on
  struct FwdGraph {
    std::vector<int> lens;
    void* ws;
    int ws_tokens, ws_seqs;
    void* pin;
    size_t pin_bytes;
    cudaGraphExec_t exec;
    uint64_t used;
  };
  std::vector<FwdGraph> graphs;
  uint64_t graph_clock = 0;
};

// drop every captured forward of d (the workspace, staging or model changed)
void graphs_clear(Device& d);

struct Global {
  std::mutex mu;
  std::mutex stat_mu;  // counters updated from per-device worker threads
  std::vector<Device*> devs;
  bool inited = false;
  size_t max_bytes = 0;  // EC_MAX_BYTES (0 = unlimited), per device
  size_t cache_bytes = size_t{24} << 30;  // EC_ALLOC_CACHE_MB: freed blocks kept per device
  int max_tokens = 262144;
  // profiling of the forward (ecdbg_profile)
  bool profile = false;
  bool sync_each = false;  // EC_SYNC_EACH_LAUNCH: wait for and report every forward launch
  ProfAcc prof[4];  // gemm, attention, rows, scan
  long long launches = 0;
  long long assign_tc_rows = 0;     // rows the tensor-core assignment settled
  long long assign_exact_rows = 0;  // rows that took the exact scan
  // multi-process communicator
  void* comm = nullptr;
  int rank = 0, world = 1;
};

Global& G();

int set_error(int code, const char* fmt, ...);
void clear_error();

// checked device allocation on the current device (honours EC_MAX_BYTES)
int dev_alloc(Device& d, void** p, size_t bytes, const char* what);
void dev_free(Device& d, void* p, size_t bytes);

int check_cuda(cudaError_t e, const char* what);
// synchronise d.stream and translate both CUDA errors and the device status
// word (bounded-wait timeouts) into a status code
int sync_and_check(Device& d, const char* what);
// Copy `bytes` of pageable host memory to device memory, enqueued on the
// device's stream after the work already there; returns once the source may
// be reused.  Large copies go through double-buffered pinned staging filled
// by several host threads, so the host copy and the DMA overlap.
int upload_h2d(Device& d, void* dst, const void* src, size_t bytes, const char* what);

struct JVal;
// build the model of config.json (+ pooling config) from d.uploads
int load_model_on(Device& d, const JVal& cfg, const JVal* pool);

// forward entry used by ec_embed_batch / ec_embed_batch_device
int embed_on_device(Device& d, const int32_t* ids_host, const int32_t* ids_dev,
                    const std::vector<int>& seqs, const int64_t* offsets, float* out_host,
                    int out_stride, float* out_dev);

// profiling helpers: bracket one launch with events (no-op unless profiling)
int prof_begin(Device& d);
void prof_end(Device& d, int cls, double flops, double bytes, int e0);
// With EC_SYNC_EACH_LAUNCH set: wait (at most 60 s) for the launch just
// enqueued and print its name, status and duration to stderr.
void trace_launch(Device& d, const char* what);
// fold finished events of d into G().prof (call after synchronising d.stream)
void prof_collect(Device& d);

// model teardown
void free_model(Device& d);
void free_index(Device& d);
// address of ec_flat_search_noalloc's static scratch array on the current
// device and context (ec_noalloc.cu); placing it loads that module
int noalloc_scratch_current(void** out);

}  // namespace ec
