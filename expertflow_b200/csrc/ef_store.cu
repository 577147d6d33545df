// ef_store.cu -- expert blobs read from model files (the cold tier below the
// slot pool's pinned host memory).
//
// The reference streams experts out of memory-mapped checkpoint files: the
// byte range of expert e of a stacked tensor is [start + e * stride,
// start + (e + 1) * stride) with stride = tensor bytes / n_experts
// (ef_deepseek_mmap.py:431-570 for GGUF, experiments/ef_v18_prefetch2.py:76-200
// for MLX safetensors, whose prefetcher reads those ranges on a thread pool so
// the page cache holds them before the expert runs).  Here the store reads the
// nine ranges of one expert (w, scales, biases of gate, up, down) straight
// into one blob of the slot pool's layout, on its own reader threads:
//  * a blob read is split into pieces of at most kPiece bytes, so one expert
//    spreads over all readers and many experts queue in FIFO order;
//  * `direct` opens the files with O_DIRECT (page-cache bypass): each piece
//    reads the 4 KiB-aligned range around it into the reader's aligned bounce
//    buffer and copies the wanted bytes out;
//  * scales / biases stored as bf16 become fp16 in place after the read; a
//    value fp16 cannot hold exactly fails the read (EF_ERR_IO) instead of
//    being rounded.
// The store is host-only (no CUDA call), so its reads run without a GPU.
#include <algorithm>
#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <fcntl.h>
#include <thread>
#include <vector>
#include <mutex>
#include <sys/stat.h>
#include <unistd.h>

namespace ef {

// One expert blob: for each projection j (gate, up, down) its w, scales and
// biases (array a = 3 j + {0, 1, 2}), each 16-byte aligned.
struct BlobLayout {
  size_t off[10];  // off[9] = used bytes
  size_t size[9];
  size_t bytes;    // off[9] rounded up to 256
};

inline BlobLayout blob_layout(const ef_moe_cfg& c) {
  BlobLayout L{};
  const size_t H = c.hidden, I = c.inter, b = c.bits;
  const size_t rows[3] = {I, I, H}, in[3] = {H, H, I};
  size_t o = 0;
  for (int j = 0; j < 3; ++j) {
    const size_t sz[3] = {rows[j] * in[j] * b / 8, rows[j] * (in[j] / 64) * 2, rows[j] * (in[j] / 64) * 2};
    for (int a = 0; a < 3; ++a) {
      L.off[3 * j + a] = o;
      L.size[3 * j + a] = sz[a];
      o += (sz[a] + 15) & ~size_t(15);
    }
  }
  L.off[9] = o;
  L.bytes = (o + 255) & ~size_t(255);
  return L;
}

// bf16 bits -> fp16 bits when the value is exact in fp16 (IEEE binary16:
// normal exponents -14..15 carry bf16's 7 mantissa bits unchanged; smaller
// magnitudes are exact only as multiples of 2^-24).  Infinities and NaNs map
// to their fp16 counterparts.  Returns false for an inexact value.
inline bool bf16_to_f16_exact(uint16_t in, uint16_t* out) {
  const uint32_t sign = (uint32_t)(in >> 15) << 15;
  const int exp = (in >> 7) & 0xff;
  const uint32_t man = in & 0x7f;
  if (exp == 0xff) {
    *out = (uint16_t)(sign | 0x7c00u | (man ? 0x200u | (man << 3) : 0u));
    return true;
  }
  if (exp == 0) {
    if (man) return false;  // bf16 subnormals lie far below fp16's range
    *out = (uint16_t)sign;
    return true;
  }
  const int e = exp - 127;
  if (e > 15) return false;
  if (e >= -14) {
    *out = (uint16_t)(sign | (uint32_t)(e + 15) << 10 | man << 3);
    return true;
  }
  // value = M * 2^(e - 7) with M = 128 + man; in units of 2^-24: k = M * 2^(e + 17)
  const uint32_t M = 128u | man;
  const int shift = -(e + 17);
  if (shift <= 0) {  // e >= -17: k = M << -shift stays below 1024 since e < -14
    *out = (uint16_t)(sign | (M << -shift));
    return true;
  }
  if (shift >= 8 || (M & ((1u << shift) - 1u))) return false;
  *out = (uint16_t)(sign | (M >> shift));
  return true;
}

constexpr size_t kPiece = 1u << 20;     // bytes per read piece (a multiple of 4 KiB)
constexpr size_t kDirectAlign = 4096;   // O_DIRECT offset / length / buffer alignment

struct ReadTicket {
  std::atomic<int> left{0};
  std::atomic<int> err{0};       // first errno (> 0), or -1: inexact bf16 value
};

struct ReadPiece {
  ReadTicket* t;
  int fd;
  bool direct;
  bool bf16;
  uint8_t* dst;
  long long off;
  size_t len;
};

}  // namespace ef

struct ef_expert_store {
  ef_moe_cfg cfg{};
  int n_layers = 0;
  ef::BlobLayout lay{};
  std::vector<int> fds;
  int direct = 0;
  std::vector<ef_file_array> arrays;  // [n_layers][9]
  std::mutex mu;
  std::condition_variable cv_job, cv_done;
  std::deque<ef::ReadPiece> q;
  std::vector<std::thread> readers;
  bool stop = false;
  std::atomic<long long> reads{0};
  std::atomic<long long> file_bytes{0};
};

namespace {

using ef::ReadPiece;
using ef::ReadTicket;

// pread until `len` bytes or end of file; returns bytes read or -errno.
long long pread_full(int fd, uint8_t* dst, size_t len, long long off) {
  size_t got = 0;
  while (got < len) {
    const ssize_t r = pread(fd, dst + got, len - got, (off_t)(off + (long long)got));
    if (r < 0) {
      if (errno == EINTR) continue;
      return -(long long)errno;
    }
    if (r == 0) break;
    got += (size_t)r;
  }
  return (long long)got;
}

int read_piece(const ReadPiece& p, uint8_t* bounce) {
  if (!p.direct) {
    const long long r = pread_full(p.fd, p.dst, p.len, p.off);
    if (r < 0) return (int)-r;
    if ((size_t)r != p.len) return EIO;
  } else {
    const long long a0 = p.off & ~(long long)(ef::kDirectAlign - 1);
    const long long end = p.off + (long long)p.len;
    const long long a1 = (end + (long long)ef::kDirectAlign - 1) & ~(long long)(ef::kDirectAlign - 1);
    const long long r = pread_full(p.fd, bounce, (size_t)(a1 - a0), a0);  // may stop short at end of file
    if (r < 0) return (int)-r;
    if (r < end - a0) return EIO;
    memcpy(p.dst, bounce + (p.off - a0), p.len);
  }
  if (p.bf16) {
    uint16_t* v = reinterpret_cast<uint16_t*>(p.dst);
    for (size_t i = 0; i < p.len / 2; ++i)
      if (!ef::bf16_to_f16_exact(v[i], &v[i])) return -1;
  }
  return 0;
}

void reader_main(ef_expert_store* S) {
  uint8_t* bounce = nullptr;
  if (S->direct && posix_memalign(reinterpret_cast<void**>(&bounce), ef::kDirectAlign, ef::kPiece + 2 * ef::kDirectAlign))
    bounce = nullptr;
  for (;;) {
    ReadPiece p;
    {
      std::unique_lock<std::mutex> lk(S->mu);
      S->cv_job.wait(lk, [S] { return S->stop || !S->q.empty(); });
      if (S->q.empty()) break;  // stop requested and nothing left
      p = S->q.front();
      S->q.pop_front();
    }
    const int e = (p.direct && !bounce) ? ENOMEM : read_piece(p, bounce);
    if (e) {
      int zero = 0;
      p.t->err.compare_exchange_strong(zero, e);
    } else {
      S->file_bytes.fetch_add((long long)p.len);
    }
    if (p.t->left.fetch_sub(1) == 1) {
      std::lock_guard<std::mutex> lk(S->mu);
      S->cv_done.notify_all();
    }
  }
  free(bounce);
}

size_t file_size(int fd) {
  struct stat st;
  return fstat(fd, &st) == 0 ? (size_t)st.st_size : 0;
}

void store_shutdown(ef_expert_store* S) {
  {
    std::lock_guard<std::mutex> lk(S->mu);
    S->stop = true;
  }
  S->cv_job.notify_all();
  for (auto& t : S->readers) t.join();
  S->readers.clear();
  for (int fd : S->fds)
    if (fd >= 0) close(fd);
  S->fds.clear();
}

}  // namespace

namespace ef {

// Queues the reads of expert e of `layer` into dst (a blob of the store's
// layout); t counts the outstanding pieces.  Returns immediately.
void store_submit(ef_expert_store* S, int layer, int e, uint8_t* dst, ReadTicket* t) {
  std::vector<ReadPiece> ps;
  for (int a = 0; a < 9; ++a) {
    const ef_file_array& fa = S->arrays[(size_t)layer * 9 + a];
    const size_t size = S->lay.size[a];
    const long long base = fa.offset + (long long)e * fa.stride;
    for (size_t o = 0; o < size; o += kPiece)
      ps.push_back(ReadPiece{t, S->fds[fa.file], S->direct != 0, fa.bf16 != 0, dst + S->lay.off[a] + o,
                             base + (long long)o, std::min(kPiece, size - o)});
  }
  t->err.store(0);
  t->left.store((int)ps.size());
  S->reads.fetch_add(1);
  {
    std::lock_guard<std::mutex> lk(S->mu);
    for (auto& p : ps) S->q.push_back(p);
  }
  S->cv_job.notify_all();
}

bool store_done(const ReadTicket* t) { return t->left.load() == 0; }

// Blocks until t's reads finish; EF_OK or EF_ERR_IO (with a message).
ef_status store_wait(ef_expert_store* S, ReadTicket* t, int layer, int e) {
  if (t->left.load() != 0) {
    std::unique_lock<std::mutex> lk(S->mu);
    S->cv_done.wait(lk, [t] { return t->left.load() == 0; });
  }
  const int err = t->err.load();
  if (err == -1) return fail(EF_ERR_IO, "layer %d expert %d: a bf16 scale/bias is not exact in fp16", layer, e);
  if (err) return fail(EF_ERR_IO, "layer %d expert %d: read failed: %s", layer, e, strerror(err));
  return EF_OK;
}

}  // namespace ef

extern "C" {

ef_status ef_store_open(const ef_moe_cfg* cfg, int n_layers, const char* const* paths, int n_files,
                        const ef_file_array* arrays, int n_readers, int direct, ef_expert_store** out) {
  if (!out) return fail(EF_ERR_INVALID, "out is NULL");
  *out = nullptr;
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (n_layers <= 0 || n_files <= 0 || !paths || !arrays) return fail(EF_ERR_INVALID, "need layers, files and arrays");
  // readers block in pread: many more than cores keep a disk's queue full (a
  // lone expert read measured 0.6 GB/s with 8 readers, 1.0-1.2 GB/s with 32-64)
  if (n_readers <= 0) n_readers = std::max(8, std::min(64, 4 * (int)std::thread::hardware_concurrency()));
  if (n_readers > 64) return fail(EF_ERR_INVALID, "n_readers must be <= 64");
  ef_expert_store* S = new ef_expert_store();
  S->cfg = *cfg;
  S->n_layers = n_layers;
  S->lay = ef::blob_layout(*cfg);
  S->direct = direct ? 1 : 0;
  S->arrays.assign(arrays, arrays + (size_t)n_layers * 9);
  std::vector<size_t> sizes;
  for (int f = 0; f < n_files; ++f) {
    if (!paths[f]) {
      store_shutdown(S);
      delete S;
      return fail(EF_ERR_INVALID, "file %d: NULL path", f);
    }
    const int fd = open(paths[f], O_RDONLY | O_CLOEXEC | (direct ? O_DIRECT : 0));
    if (fd < 0) {
      const int e = errno;
      store_shutdown(S);
      delete S;
      return fail(EF_ERR_IO, "%s: cannot open%s: %s", paths[f], direct ? " with O_DIRECT" : "", strerror(e));
    }
    S->fds.push_back(fd);
    sizes.push_back(file_size(fd));
  }
  const long long E = cfg->n_experts;
  for (int l = 0; l < n_layers; ++l) {
    for (int a = 0; a < 9; ++a) {
      const ef_file_array& fa = S->arrays[(size_t)l * 9 + a];
      const long long size = (long long)S->lay.size[a];
      const char* why = nullptr;
      if (fa.file < 0 || fa.file >= n_files) why = "file index out of range";
      else if (fa.offset < 0 || fa.stride < size) why = "offset < 0 or stride below the array size";
      else if (fa.offset + (E - 1) * fa.stride + size > (long long)sizes[fa.file]) why = "expert ranges run past the end of the file";
      else if (fa.bf16 && a % 3 == 0) why = "codes cannot be bf16";
      else if (fa.bf16 && ((fa.offset | fa.stride) & 1)) why = "bf16 array not 2-byte aligned";
      if (why) {
        store_shutdown(S);
        delete S;
        return fail(EF_ERR_INVALID, "layer %d array %d: %s", l, a, why);
      }
    }
  }
  for (int i = 0; i < n_readers; ++i) S->readers.emplace_back(reader_main, S);
  *out = S;
  return EF_OK;
}

ef_status ef_store_get_info(const ef_expert_store* S, ef_store_info* out) {
  if (!S || !out) return fail(EF_ERR_INVALID, "null pointer");
  out->blob_bytes = S->lay.bytes;
  for (int a = 0; a < 10; ++a) out->offsets[a] = S->lay.off[a];
  out->n_layers = S->n_layers;
  out->n_readers = (int)S->readers.size();
  out->direct = S->direct;
  out->reads = S->reads.load();
  out->file_bytes = (double)S->file_bytes.load();
  return EF_OK;
}

ef_status ef_store_read(ef_expert_store* S, int n, const int32_t* layers, const int32_t* experts, void* const* dst) {
  if (!S) return fail(EF_ERR_INVALID, "store is NULL");
  if (n < 0 || (n && (!layers || !experts || !dst))) return fail(EF_ERR_INVALID, "null pointer");
  for (int i = 0; i < n; ++i) {
    if (layers[i] < 0 || layers[i] >= S->n_layers || experts[i] < 0 || experts[i] >= S->cfg.n_experts)
      return fail(EF_ERR_RANGE, "read %d: layer %d expert %d out of range", i, layers[i], experts[i]);
    if (!dst[i]) return fail(EF_ERR_INVALID, "read %d: NULL destination", i);
  }
  std::vector<ReadTicket> t(n);
  for (int i = 0; i < n; ++i) ef::store_submit(S, layers[i], experts[i], static_cast<uint8_t*>(dst[i]), &t[i]);
  ef_status first = EF_OK;
  for (int i = 0; i < n; ++i) {
    const ef_status s = ef::store_wait(S, &t[i], layers[i], experts[i]);
    if (s && !first) first = s;
  }
  return first;
}

ef_status ef_store_close(ef_expert_store* S) {
  if (!S) return EF_OK;
  store_shutdown(S);
  delete S;
  return EF_OK;
}

}  // extern "C"
