// ec_files.cu -- the on-disk formats of the index path, read and written in
// the library so that a host never copies them through its own arrays:
//
//   index.bin  rows of `dim` little-endian f32, no header (embed::write-f32,
//              embed.lisp:47-57; read by ann::load-vectors, ann.lisp:37-55,
//              and kb::load-index, kb.lisp:84-129);
//   ann.bin    u32 0x414E4E31 ("ANN1"), u32 k, u32 dim, u32 n, then k*dim
//              f32 centroids, k u32 counts, n u32 row ids grouped by centroid
//              (ann::save-ann, ann.lisp:165-187; kb::load-ann, kb.lisp:283-314).
//
// The dimension is a parameter throughout; the reference takes it from the
// constant 384 (ann.lisp:19, kb.lisp:23, embed.lisp:83).  index.bin is mapped
// read-only and uploaded from the mapping (upload_h2d stages it through pinned
// buffers), so the 4 B x n x dim vectors are never copied into a host array.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <vector>

#include "ec_state.h"

namespace ec {
namespace {

constexpr uint32_t kAnnMagic = 0x414E4E31u;

// read-only mapping of a whole file
struct MappedFile {
  void* p = MAP_FAILED;
  size_t n = 0;
  int fd = -1;
  int open(const char* path) {
    fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(EC_EINVAL, "cannot open %s", path);
    struct stat stt;
    if (fstat(fd, &stt) != 0) return set_error(EC_EINVAL, "cannot stat %s", path);
    n = static_cast<size_t>(stt.st_size);
    if (n == 0) return set_error(EC_EINVAL, "%s is empty", path);
    p = mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) return set_error(EC_EINVAL, "cannot map %s", path);
    return EC_OK;
  }
  ~MappedFile() {
    if (p != MAP_FAILED) munmap(p, n);
    if (fd >= 0) ::close(fd);
  }
};

static void put_u32(unsigned char* b, uint32_t v) {
  b[0] = static_cast<unsigned char>(v);
  b[1] = static_cast<unsigned char>(v >> 8);
  b[2] = static_cast<unsigned char>(v >> 16);
  b[3] = static_cast<unsigned char>(v >> 24);
}
static uint32_t get_u32(const unsigned char* b) {
  return static_cast<uint32_t>(b[0]) | (static_cast<uint32_t>(b[1]) << 8) |
         (static_cast<uint32_t>(b[2]) << 16) | (static_cast<uint32_t>(b[3]) << 24);
}

static int write_all(FILE* f, const void* p, size_t bytes, const char* path) {
  if (bytes && fwrite(p, 1, bytes, f) != bytes) return set_error(EC_EINVAL, "short write to %s", path);
  return EC_OK;
}

// index.bin rows of dimension d: n rows, or an error if the size does not fit
static int index_rows(const MappedFile& m, int d, const char* path, int64_t* n) {
  const size_t row = static_cast<size_t>(d) * 4;
  if (m.n % row) return set_error(EC_EINVAL, "%s: %zu bytes is not a multiple of %d f32 rows", path, m.n, d);
  *n = static_cast<int64_t>(m.n / row);
  return EC_OK;
}

}  // namespace
}  // namespace ec

using namespace ec;

extern "C" {

int ec_ann_save(const char* path, const float* centroids, int k, int d, int64_t n,
                const uint32_t* counts, const uint32_t* lists) {
  clear_error();
  if (!path || !centroids || !counts || (n > 0 && !lists) || k <= 0 || d <= 0 || n < 0 ||
      n > 0xffffffffll)
    return set_error(EC_EINVAL, "bad ann.bin arguments");
  uint64_t total = 0;
  for (int c = 0; c < k; ++c) total += counts[c];
  if (total != static_cast<uint64_t>(n))
    return set_error(EC_EINVAL, "counts sum to %llu, not n = %lld", static_cast<unsigned long long>(total),
                     static_cast<long long>(n));
  FILE* f = fopen(path, "wb");
  if (!f) return set_error(EC_EINVAL, "cannot create %s", path);
  unsigned char hdr[16];
  put_u32(hdr, kAnnMagic);
  put_u32(hdr + 4, static_cast<uint32_t>(k));
  put_u32(hdr + 8, static_cast<uint32_t>(d));
  put_u32(hdr + 12, static_cast<uint32_t>(n));
  // the arrays are written as they lie in memory: this library runs on
  // little-endian hosts only (x86-64, aarch64), like the reference's files
  int rc = write_all(f, hdr, 16, path);
  if (!rc) rc = write_all(f, centroids, static_cast<size_t>(k) * d * 4, path);
  if (!rc) rc = write_all(f, counts, static_cast<size_t>(k) * 4, path);
  if (!rc) rc = write_all(f, lists, static_cast<size_t>(n) * 4, path);
  if (fclose(f) != 0 && !rc) rc = set_error(EC_EINVAL, "cannot close %s", path);
  return rc;
}

int ec_ann_read(const char* path, int* k, int* d, int64_t* n, float* centroids, uint32_t* counts,
                uint32_t* lists) {
  clear_error();
  if (!path || !k || !d || !n) return set_error(EC_EINVAL, "bad ann.bin arguments");
  MappedFile m;
  int rc = m.open(path);
  if (rc) return rc;
  const unsigned char* b = static_cast<const unsigned char*>(m.p);
  if (m.n < 16 || get_u32(b) != kAnnMagic) return set_error(EC_EINVAL, "%s: not an ann.bin (magic)", path);
  const uint32_t kk = get_u32(b + 4), dd = get_u32(b + 8), nn = get_u32(b + 12);
  // k x d is checked against the file before the total is formed, so a
  // header with huge sizes cannot wrap the total around to the file's size
  if (kk == 0 || dd == 0 || kk > 0x7fffffffu || dd > 0x7fffffffu ||
      static_cast<uint64_t>(kk) * dd > m.n / 4)
    return set_error(EC_EINVAL, "%s: %zu bytes, header says k %u x dim %u", path, m.n, kk, dd);
  const size_t need = 16 + (static_cast<size_t>(kk) * dd + kk + nn) * 4;
  if (m.n != need) return set_error(EC_EINVAL, "%s: %zu bytes, header says %zu", path, m.n, need);
  *k = static_cast<int>(kk);
  *d = static_cast<int>(dd);
  *n = nn;
  size_t o = 16;
  if (centroids) std::memcpy(centroids, b + o, static_cast<size_t>(kk) * dd * 4);
  o += static_cast<size_t>(kk) * dd * 4;
  if (counts) std::memcpy(counts, b + o, static_cast<size_t>(kk) * 4);
  o += static_cast<size_t>(kk) * 4;
  if (lists) std::memcpy(lists, b + o, static_cast<size_t>(nn) * 4);
  return EC_OK;
}

int ec_index_load_files(const char* index_path, int d, const char* ann_path, int64_t* n_out) {
  clear_error();
  if (!index_path || d <= 0) return set_error(EC_EINVAL, "bad index file arguments");
  MappedFile m;
  int rc = m.open(index_path);
  if (rc) return rc;
  int64_t n = 0;
  if ((rc = index_rows(m, d, index_path, &n))) return rc;
  if (n_out) *n_out = n;
  if (!ann_path) return ec_index_load(static_cast<const float*>(m.p), n, d, nullptr, 0, nullptr, nullptr);
  int k = 0, ad = 0;
  int64_t an = 0;
  if ((rc = ec_ann_read(ann_path, &k, &ad, &an, nullptr, nullptr, nullptr))) return rc;
  if (ad != d || an != n)
    return set_error(EC_EINVAL, "%s is for %lld rows of dim %d, %s has %lld rows of dim %d", ann_path,
                     static_cast<long long>(an), ad, index_path, static_cast<long long>(n), d);
  std::vector<float> cent(static_cast<size_t>(k) * d);
  std::vector<uint32_t> counts(k), lists(static_cast<size_t>(n));
  if ((rc = ec_ann_read(ann_path, &k, &ad, &an, cent.data(), counts.data(), lists.data()))) return rc;
  return ec_index_load(static_cast<const float*>(m.p), n, d, cent.data(), k, counts.data(),
                       lists.data());
}

int ec_ann_build_file(const char* index_path, int d, int k, int iters, const int64_t* sample,
                      int64_t nsample, const char* ann_path) {
  clear_error();
  if (!index_path || !ann_path || d <= 0 || k <= 0 || iters < 0 || !sample || nsample < k)
    return set_error(EC_EINVAL, "bad ann build arguments");
  MappedFile m;
  int rc = m.open(index_path);
  if (rc) return rc;
  int64_t n = 0;
  if ((rc = index_rows(m, d, index_path, &n))) return rc;
  const float* x = static_cast<const float*>(m.p);
  std::vector<float> cent(static_cast<size_t>(k) * d);
  std::vector<uint32_t> counts(k), lists(static_cast<size_t>(n));
  rc = ec_ann_build(x, n, d, sample, nsample, k, iters, nullptr, cent.data(), counts.data(),
                    lists.data());
  if (rc) return rc;
  return ec_ann_save(ann_path, cent.data(), k, d, n, counts.data(), lists.data());
}

int ec_embed_batch_to_file(const int32_t* ids, const int64_t* offsets, int nseq,
                           const char* index_path) {
  clear_error();
  if (!index_path || nseq <= 0) return set_error(EC_EINVAL, "bad embed-to-file arguments");
  const int dim = ec_dim();
  if (dim <= 0) return dim;
  std::vector<float> out(static_cast<size_t>(nseq) * dim);
  int rc = ec_embed_batch(ids, offsets, nseq, out.data(), dim);
  if (rc) return rc;
  FILE* f = fopen(index_path, "ab");
  if (!f) return set_error(EC_EINVAL, "cannot open %s for appending", index_path);
  rc = write_all(f, out.data(), out.size() * 4, index_path);
  if (fclose(f) != 0 && !rc) rc = set_error(EC_EINVAL, "cannot close %s", index_path);
  return rc;
}

}  // extern "C"
