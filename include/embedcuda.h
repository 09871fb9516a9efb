/* embedcuda.h -- C ABI of libembedcuda.so, the B200 (sm_100a) backend of
 * lisp-embed's embedding hot path.
 *
 * Every entry point takes plain C types (pointers + sizes), returns an int
 * status (EC_OK or a negative EC_E* code) and never exits the process; the
 * message of the last failure on the calling thread is ec_last_error().
 * Host buffers belong to the caller and are only read or written during the
 * call; device memory belongs to the library.  Calls are serialised by an
 * internal mutex, so the many sb-thread workers of embed.lisp may call in
 * concurrently.
 *
 * Each declaration cites the reference function it stands in for
 * (file:line in drvova/lisp-embed).
 */
#ifndef EMBEDCUDA_H
#define EMBEDCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
#define EC_OK 0
#define EC_EINVAL (-1)    /* bad argument, shape or dtype                      */
#define EC_ESTATE (-2)    /* call out of order (no ec_init / no model / index) */
#define EC_ECUDA (-3)     /* CUDA runtime or driver error                      */
#define EC_ENOMEM (-4)    /* device allocation failed or over EC_MAX_BYTES     */
#define EC_ETIMEOUT (-5)  /* a kernel's bounded wait ran out (kernel aborted)  */
#define EC_ENCCL (-6)     /* NCCL missing or a collective failed               */
#define EC_EUNSUPPORTED (-7) /* model family / config outside this build      */

/* ---- dtypes of ec_upload_tensor (safetensors "dtype") ----------------------- */
#define EC_F32 0
#define EC_BF16 1
#define EC_F16 2

/* ---- model families returned by ec_load_model (model.lisp:11) -------------- */
#define EC_FAMILY_BERT 1   /* bert / roberta / distilbert (bert.lisp)        */
#define EC_FAMILY_MPNET 2  /* mpnet (bert.lisp:322-499)                      */
#define EC_FAMILY_LLAMA 3  /* llama / qwen2 / qwen3 / mistral (llama.lisp)    */
#define EC_FAMILY_GEMMA 4  /* embedding_gemma2 (gemma.lisp)                    */

/* Message of the last failed call on this thread ("" if none). */
const char *ec_last_error(void);

/* Bring up the library on `ndev` CUDA devices listed in `devices` (NULL or
 * ndev <= 0: the devices named by EC_DEVICES, else every visible device).
 * Replaces nothing in the reference: it is the GPU context that the Lisp
 * globals of model.lisp:11-12 and bert.lisp:10-27 stand for. */
int ec_init(const int *devices, int ndev);

/* Number of devices the library drives (after ec_init). */
int ec_device_count(void);

/* Release every device buffer, stream and communicator. */
int ec_shutdown(void);

/* Upload one safetensors tensor with its raw bytes (no host widening) to every
 * device.  Replaces st:get-tensor (st.lisp:32-86): F32 is kept bit-exact,
 * BF16 and F16 are widened on the device with st.lisp's rules (BF16 << 16;
 * F16 exponent 31 -> +-most-positive-single-float, st.lisp:29). */
int ec_upload_tensor(const char *name, int dtype, const int64_t *shape, int ndim,
                     const void *data, size_t nbytes);

/* Build the model from the uploaded tensors.  `config_json` is config.json,
 * `pooling_json` is 1_Pooling/config.json or NULL.  Replaces
 * model:load-model's dispatch (model.lisp:28-46) plus bert:load-model
 * (bert.lisp:55-129, 343-389), llama:load-model (llama.lisp:172-220) and
 * gemma:load-model (gemma.lisp:140-212).
 * Writes the family (EC_FAMILY_*) and the embedding dimension. */
int ec_load_model(const char *config_json, const char *pooling_json, int *family,
                  int *dim);

/* Embedding dimension of the loaded model; replaces model:dim (model.lisp:56-62).
 * Returns the dimension (> 0) or a negative status. */
int ec_dim(void);

/* Embed `nseq` token-id sequences.  Sequence s is ids[offsets[s] ..
 * offsets[s+1]); `out` receives nseq rows of ec_dim() floats at a stride of
 * `out_stride` floats, L2-normalised, in input order.  Replaces model:embed
 * (model.lisp:48-54) -> bert::embed-bert (bert.lisp:275-320),
 * bert::embed-mpnet (:455-499), llama:embed (llama.lisp:296-344) and
 * gemma:embed (gemma.lisp:306-380) for a whole batch, the way embed:run
 * batches chunks (embed.lisp:88-105).  offsets must ascend from >= 0, every
 * sequence hold 1 .. the model's positions ids, every id lie in the
 * vocabulary; otherwise EC_EINVAL before anything is computed.  The library
 * cannot see the length of ids: offsets[nseq] must not pass it. */
int ec_embed_batch(const int32_t *ids, const int64_t *offsets, int nseq, float *out,
                   int out_stride);

/* Device-resident variant for callers that keep ids and outputs in HBM
 * (single device only): `d_ids` and `d_out` are device pointers on the
 * library's device 0; `offsets` stays on the host.  The work is enqueued on
 * `stream` (a cudaStream_t; NULL = the library's own stream) after the work
 * already queued there, and the call returns once it has finished.  Same
 * semantics as ec_embed_batch. */
int ec_embed_batch_device(const int32_t *d_ids, const int64_t *offsets, int nseq,
                          float *d_out, int out_stride, void *stream);

/* ---- IVF (ann.lisp, kb.lisp) ------------------------------------------------- */

/* Lloyd k-means over the rows of x (n x d, row-major f32).  The training set
 * is x[sample[0..nsample)] in that order and centroid c starts as
 * x[sample[c]] (ann.lisp:83-86), or as init[c] when `init` is not NULL.  Each iteration assigns every training row
 * to its nearest centroid by inner product (ties -> lowest index,
 * ann.lisp:69-77) and replaces each non-empty centroid by the mean of its
 * rows (ann.lisp:107-122).  The training set is split into contiguous
 * shards, one per device (or per process after ec_comm_init, where rank r
 * passes the r-th contiguous piece of the sample).  Each rank assigns its
 * shard; the per-cluster sums then pass down the ranks in sample order over
 * NCCL (rank r continues rank r-1's accumulators with its own rows) and the
 * last rank divides and broadcasts the centroids, so every float add follows
 * the reference's serial loop and the result does not depend on the number
 * of devices.  EC_KMEANS_ALLREDUCE=1 instead all-reduces per-rank sums (one
 * ncclAllReduce per iteration; the cross-rank sums then take another order).
 * A failed exchange aborts the communicators (process mode: call
 * ec_comm_init again).  `centroids` receives k x d floats.  Replaces
 * ann::kmeans (ann.lisp:79-125). */
int ec_kmeans(const float *x, int64_t n, int d, const int64_t *sample, int64_t nsample,
              int k, int iters, const float *init, float *centroids);

/* Assign every row of x to its nearest centroid and build the inverted lists:
 * counts[k] and lists[n] (row ids grouped by centroid, ascending within each
 * list).  Replaces ann::assign-all (ann.lisp:127-158). */
int ec_assign_all(const float *x, int64_t n, int d, const float *centroids, int k,
                  uint32_t *counts, uint32_t *lists);

/* ec_kmeans followed by ec_assign_all with its centroids, as ann:run does
 * (ann.lisp:193-197): the same arguments and results as the two calls, but
 * on one device the rows cross to it once (the sample's rows are gathered
 * from that copy on the device, and the final assignment reuses it).  With
 * several devices in the process it makes the two calls.  Replaces the
 * kmeans + assign-all pair of ann:run (ann.lisp:189-200). */
int ec_ann_build(const float *x, int64_t n, int d, const int64_t *sample, int64_t nsample,
                 int k, int iters, const float *init, float *centroids, uint32_t *counts,
                 uint32_t *lists);

/* One assignment pass with explicit centroids: assign[i] = nearest centroid
 * of x[rows[i]] (rows NULL: row i).  Replaces the assign step of ann::kmeans
 * (ann.lisp:90-105). */
int ec_assign(const float *x, int64_t n, int d, const int64_t *rows, int64_t nrows,
              const float *centroids, int k, int32_t *assign);

/* Keep an index resident on the devices: vectors (n x d), centroids (k x d),
 * counts[k], lists[n] -- the contents of index.bin and ann.bin.  Replaces
 * kb::load-index's vector part (kb.lisp:84-129) and kb::load-ann
 * (kb.lisp:283-314).  k = 0 loads vectors only (flat search). */
int ec_index_load(const float *x, int64_t n, int d, const float *centroids, int k,
                  const uint32_t *counts, const uint32_t *lists);

/* IVF search of nq queries (nq x d): the nprobe best centroids by inner
 * product, exact scan of their lists, top `topk` by score (descending).
 * ids[nq x topk] / scores[nq x topk]; unused slots get id -1.  Results equal
 * kb::top-k-ivf (kb.lisp:348-364), ties broken as its stable sorts do. */
int ec_ivf_search(const float *q, int nq, int nprobe, int topk, int64_t *ids,
                  float *scores);

/* Exact flat search over all resident vectors; replaces kb::top-k-brute
 * (kb.lisp:186-200).  Ties -> lower row id first. */
int ec_flat_search(const float *q, int nq, int topk, int64_t *ids, float *scores);

/* Flat search like ec_flat_search, over caller-owned DEVICE buffers on the
 * current device, that allocates no device memory (no counterpart in the
 * reference: kb::top-k-brute, kb.lisp:186-200, always allocates).  For hosts
 * that cannot let the library allocate mid-request: an image that reserves
 * its device arena up front (the allocation would fail once the arena is
 * taken) or a request loop that cannot absorb the device-wide synchronisation
 * cudaMalloc / cudaFree may cause.  d_x: n x d vectors, d_q: nq x d queries
 * (both 16-byte aligned, d % 4 == 0, d <= 8192, 0 < n < 2^31), d_ids /
 * d_scores: nq x topk (1 <= topk <= 64), same order and ties as
 * ec_flat_search.  Enqueued on `stream` (a cudaStream_t, NULL = legacy
 * default stream) and not synchronised.  The candidate lists live in one
 * static 16 MiB device array per device: a call needs
 * nq x min(256, ceil(n / 8192)) x topk x 8 bytes of it (nq <= 65535) and
 * larger calls fail with EC_EINVAL before any launch.  Every call on a device
 * shares that array, so calls whose kernels overlap in time race; calls in
 * order on one stream do not.  The array is placed in device memory when
 * the library's module holding it loads on a device: at ec_init for the
 * library's devices, otherwise at the first call with nq > 0 (CUDA loads
 * modules lazily), so a host that reserves its device arena up front should
 * call ec_init, or make one search, before it takes the arena.  The first
 * call in each CUDA context looks up the array's address (cached per device
 * and context), so make it before any stream capture begins.  Needs no
 * ec_init. */
int ec_flat_search_noalloc(const float *d_x, int64_t n, int d, const float *d_q, int nq,
                           int topk, int64_t *d_ids, float *d_scores, void *stream);

/* ---- index files (no reference counterpart in C; the formats are the
 * reference's, with the dimension passed in instead of the constant 384 of
 * ann.lisp:19 / kb.lisp:23 / embed.lisp:83) --------------------------------- */

/* Write ann.bin: u32 0x414E4E31, k, dim, n; k x dim f32 centroids; k u32
 * counts; n u32 row ids grouped by centroid.  Same bytes as ann::save-ann
 * (ann.lisp:165-187).  counts must sum to n.  Needs no ec_init. */
int ec_ann_save(const char *path, const float *centroids, int k, int d, int64_t n,
                const uint32_t *counts, const uint32_t *lists);

/* Read ann.bin (kb::load-ann, kb.lisp:283-314): writes k, d and n; fills the
 * arrays that are not NULL (k x d, k, n elements).  A wrong magic or size is
 * EC_EINVAL.  Needs no ec_init. */
int ec_ann_read(const char *path, int *k, int *d, int64_t *n, float *centroids,
                uint32_t *counts, uint32_t *lists);

/* Make index.bin (rows of d f32, n = file size / 4d) and, when ann_path is not
 * NULL, ann.bin resident on every device, reading the vectors from a mapping
 * of the file (no host copy).  Replaces the vector and ann parts of
 * kb::load-index (kb.lisp:84-129) and kb::load-ann (kb.lisp:283-314); same
 * state as ec_index_load afterwards.  Writes n (may be NULL). */
int ec_index_load_files(const char *index_path, int d, const char *ann_path, int64_t *n);

/* ann:run from index.bin to ann.bin (ann.lisp:189-200): k-means over the rows
 * sample[0..nsample) (centroids start at the first k of them), then
 * assign-all and ann.bin.  The sample is explicit: the reference draws it
 * with SBCL's random state (ann.lisp:57-67). */
int ec_ann_build_file(const char *index_path, int d, int k, int iters, const int64_t *sample,
                      int64_t nsample, const char *ann_path);

/* ec_embed_batch, then the rows appended to index.bin the way embed:run
 * writes them (embed.lisp:47-57, 99-101): ec_dim() f32 per sequence, input
 * order. */
int ec_embed_batch_to_file(const int32_t *ids, const int64_t *offsets, int nseq,
                           const char *index_path);

/* ---- tokenizer (tokenizer.lisp) ----------------------------------------------
 * Host-only (no GPU, no ec_init).  A tokenizer is a handle > 0; it is
 * read-only after loading, so any number of threads may tokenize with it. */

/* make-tokenizer-from-json (tokenizer.lisp:515-552): HF tokenizer.json with a
 * WordPiece or BPE model; specials from the post-processor (json-specials,
 * :465-498), pre-tokenizer family from its regex (pretok-mode, :500-513). */
int ec_tokenizer_from_json(const char *path, int *handle);
/* make-tokenizer :wordpiece (tokenizer.lisp:126-140, bert.lisp:45): vocab.txt,
 * one token per line, id = line number. */
int ec_tokenizer_wordpiece(const char *vocab_txt, int lowercase, int *handle);
/* make-tokenizer :bpe (tokenizer.lisp:141-173; bert.lisp:47-53, llama.lisp:76-80):
 * vocab.json + merges.txt.  NULL special-token names keep the defaults
 * "[CLS]", "[SEP]", "[UNK]"; bos_id / eos_id < 0: none. */
int ec_tokenizer_bpe(const char *vocab_json, const char *merges_txt, int lowercase,
                     int byte_level, int llama3, const char *cls_token, const char *sep_token,
                     const char *unk_token, int bos_id, int eos_id, int *handle);
/* make-tokenizer :unigram (tokenizer.lisp:174-197): {token: log score}. */
int ec_tokenizer_unigram(const char *scores_json, int lowercase, int *handle);
int ec_tokenizer_free(int handle);
/* Number of ids of the vocabulary (tk-vocab-size, tokenizer.lisp:254). */
int ec_tokenizer_vocab_size(int handle);
/* tk-encode (tokenizer.lisp:201-244) of ntexts UTF-8 texts (texts[i] of
 * lengths[i] bytes, or NUL-terminated when lengths is NULL; a NULL texts[i]
 * only with lengths[i] == 0, an empty text; a NULL text otherwise or a
 * negative length is EC_EINVAL) on nthreads host
 * threads (<= 0: all cores).  Ids are packed into ids[0..offsets[ntexts]) with
 * text i at [offsets[i], offsets[i+1]) -- the layout ec_embed_batch takes.
 * Each text yields at most 512 ids.  If they do not fit `cap`, the call fails
 * with EC_EINVAL after filling offsets (offsets[ntexts] = the count needed). */
int ec_tokenize(int handle, const char *const *texts, const int64_t *lengths, int ntexts,
                int32_t *ids, int64_t cap, int64_t *offsets, int nthreads);
/* tk-decode (tokenizer.lisp:246-252): the tokens of ids concatenated into
 * out (UTF-8, not NUL-terminated); *len = the byte count. */
int ec_tokenizer_decode(int handle, const int32_t *ids, int n, char *out, int64_t cap,
                        int64_t *len);

/* ---- multi-process (one process per GPU) ------------------------------------ */

/* Size of the opaque NCCL unique id (128 bytes). */
int ec_comm_id_size(void);
/* Rank 0 creates the id; the caller ships it to the other ranks. */
int ec_comm_get_id(void *id_out);
/* Join a `world`-rank communicator as `rank` (after ec_init on one device).
 * ec_kmeans then exchanges across processes instead of local devices: rank r
 * passes the r-th contiguous piece of the training sample (in sample order)
 * and every rank the same `init`. */
int ec_comm_init(int rank, int world, const void *id);

#ifdef __cplusplus
}
#endif
#endif /* EMBEDCUDA_H */
