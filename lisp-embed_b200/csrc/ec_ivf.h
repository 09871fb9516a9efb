// ec_ivf.h -- launchers of the IVF kernels (ec_ivf_kernels.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ec {

// assign[i] = argmax_c <X[rows ? rows[i] : i], C[c]>, ties -> lowest c
cudaError_t launch_assign(const float* X, const int64_t* rows, int64_t n, const float* C, int k,
                          int d, int32_t* out, cudaStream_t st);
// S[q, c] = <Q[q], C[c]> (sequential single-float order)
cudaError_t launch_scores(const float* Q, int64_t nq, const float* C, int k, int d, float* S,
                          cudaStream_t st, unsigned* status = nullptr);
// stable counting sort of assignments into inverted lists:
// counts[k], offs[k + 1], lists[n] (base + row id, ascending within a list);
// tile_hist needs sort_tiles(n) * k words of scratch
int64_t sort_tiles(int64_t n);
cudaError_t launch_lists(const int32_t* a, int64_t n, int k, uint32_t* tile_hist,
                         uint32_t* counts, int64_t* offs, uint32_t base, uint32_t* lists,
                         cudaStream_t st);
// out[c * (d + 1) + j] = sum of X[list c][j] in list order; [.. + d] = count;
// with `init` (same layout) the sums and counts continue from init's values
cudaError_t launch_segsum(const float* X, const uint32_t* lists, const int64_t* offs, int k,
                          int d, const float* init, float* out, cudaStream_t st);
cudaError_t launch_update(const float* sums, int k, int d, float* cent, cudaStream_t st);
cudaError_t launch_probe_select(const float* S, int64_t nq, int k, int nprobe, int32_t* probes,
                                cudaStream_t st);
// the same probes from tensor-core scores S (|S - exact| <= rel2 |q| max|c| / 2):
// candidates within the window re-scored exactly; Q, C the fp32 queries and
// centroids, qnorm / cmax upper bounds of their norms
cudaError_t launch_probe_select_tc(const float* S, const float* Q, const float* C, const float* qnorm,
                                   const float* cmax, float rel2, int64_t nq, int k, int d, int nprobe,
                                   int32_t* probes, cudaStream_t st);
// one CTA per (query, probed list, part): each list split into `parts`
// contiguous pieces, candidates [nq][nprobe][parts][topk]
cudaError_t launch_list_scan(const float* X, int d, const uint32_t* lists, const int64_t* offs,
                             const int32_t* probes, int nprobe, const float* Q, int64_t nq,
                             int topk, int parts, unsigned long long* cand, cudaStream_t st,
                             unsigned* status = nullptr);
cudaError_t launch_flat_scan(const float* X, int64_t n, int d, int nchunks, const float* Q,
                             int64_t nq, int topk, unsigned long long* cand, cudaStream_t st);
cudaError_t launch_merge(const unsigned long long* cand, int64_t nq, int ngroups, int topk,
                         int64_t* ids, float* scores, cudaStream_t st);

// ---- query-batched scans (ec_ivf_scan.cu): same candidates as
// launch_list_scan / launch_flat_scan, one CTA per (list or row chunk, up to
// 32 queries).  Needs d % 4 == 0, 16-byte aligned X and Q, topk <= 64.
bool batched_scan_supported(const float* X, const float* Q, int d, int topk);
// bytes of scratch launch_list_scan_batched needs
size_t batched_list_scan_ws(int k, int64_t npairs);
cudaError_t launch_list_scan_batched(const float* X, int d, const uint32_t* lists,
                                     const int64_t* offs, int k, const int32_t* probes, int nprobe,
                                     const float* Q, int64_t nq, int topk, void* ws,
                                     unsigned long long* cand, cudaStream_t st);
cudaError_t launch_flat_scan_batched(const float* X, int64_t n, int d, int nchunks,
                                     const float* Q, int64_t nq, int topk,
                                     unsigned long long* cand, cudaStream_t st);

// ---- tensor-core assignment (ec_ivf_tc.cu) ----------------------------------
// relative bound on |bf16 score - exact score| / (|x| max|c|) for head dim d
float argcand_rel(int d);
// Xb = bf16(X) [n, d]; norms[r] >= |X[r]| (nullptr: skip); *nmax >= the
// largest (nullptr: skip; the caller zeroes it first)
cudaError_t launch_round_rows(const float* X, int64_t n, int d, __nv_bfloat16* Xb, float* norms,
                              unsigned* nmax, cudaStream_t st);
// exact argmax over each row's candidate columns (the kEpiArgCand GEMM's
// output, `parts` column parts); rows that need the exact scan are appended
// to fb_rows / *fb_count instead
cudaError_t launch_argcand_reduce(const float* X, int64_t n, int d, const float* C,
                                  const float* xnorm, const float* cmax, float rel2, int parts,
                                  const float* mloc, const uint32_t* pk, int32_t* out,
                                  int64_t* fb_rows,
                                  unsigned long long* fb_count, cudaStream_t st);
// out[j] = X[rows[j]] for j < m (rows of d floats, d % 4 == 0; the caller
// checks every index against X's rows)
cudaError_t launch_gather_rows(const float* X, const int64_t* rows, int64_t m, int d, float* out,
                               int num_sms, cudaStream_t st);
// out[fb_rows[i]] = vals[i]
cudaError_t launch_scatter_assign(const int64_t* fb_rows, int64_t nfb, const int32_t* vals,
                                  int32_t* out, cudaStream_t st);

}  // namespace ec
