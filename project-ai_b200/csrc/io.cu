// Native I/O paths of the training loop: PAICKPT2 checkpoints and packed token datasets.
//
// Checkpoints (ProjectAI.Formats/Checkpoint.cs:11-110, the layout kept byte for byte):
//   magic "PAICKPT2" | int32 step | int32 metaLen | metadata (UTF-8) | int32 tensorCount
//   per tensor: int32 nameLen | name | int32 rank | rank x int32 dims | int64 byteLen | f32 little-endian payload
// Save copies the tensors once into a device snapshot on the compute stream (the only work the caller's next ops
// queue behind: HBM to HBM), then a writer thread streams the snapshot to the file through two pinned host chunks on
// a copy stream of its own, so the device-to-host copy of one chunk overlaps the file write of the previous one and
// training continues meanwhile; pai_ckpt_wait joins the writer. Without room for a snapshot the save streams from the
// tensors themselves and returns when the file is written. Load walks the file with the reference's checks, reading
// chunk k+1 from the file while chunk k crosses to the device.
//
// Packed datasets (ProjectAI.Training/PackedBinDataset.cs:43-117): the shard is memory-mapped; a batch gathers its
// blocks (seq_len + 1 ids each) into pinned memory at the shard's own width (2 or 4 bytes per id), uploads them with one
// copy, and one kernel writes the F32 input and target ids the embedding and loss take (Training.cs:122-141), in place
// of widening every id to float on the host and uploading two float arrays.
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace pai {

constexpr size_t kIoChunk = size_t(32) << 20;  // pinned staging chunk for checkpoint payloads (two of them)
constexpr int32_t kMaxMeta = 1 << 24;          // Checkpoint.cs:70 / :128
constexpr int32_t kMaxName = 1 << 20;          // Checkpoint.cs:77

struct IoState {
  cudaStream_t stream = nullptr;  // copy stream for checkpoint payloads
  char* pinned = nullptr;         // two kIoChunk buffers
  cudaEvent_t ev[2] = {};
  cudaEvent_t mark = nullptr;     // a point of the compute stream (copies start after it) or of the copy stream
  // the save in flight
  std::thread writer;
  bool writing = false;
  void* snapshot = nullptr;       // device copy of the saved tensors; released after the writer joins
  pai_status save_status = PAI_OK;
  std::string save_error;
  // the last loaded checkpoint
  std::string meta;
  std::vector<std::string> names;
  std::vector<pai_tensor> tensors;
  // the open packed dataset
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t map_bytes = 0;
  int elem = 0, seq = 0;
  int64_t blocks = 0;
  char* ds_pinned[2] = {nullptr, nullptr};
  size_t ds_cap = 0;
  cudaEvent_t ds_ev[2] = {};
  int ds_next = 0;
};

static pai_status io_state(pai_ctx* ctx, IoState** out) {
  if (!ctx->io) {
    auto* s = new IoState();
    cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&s->pinned), 2 * kIoChunk, cudaHostAllocDefault);
    for (int i = 0; i < 2 && e == cudaSuccess; i++) e = cudaEventCreateWithFlags(&s->ev[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->mark, cudaEventDisableTiming);
    for (int i = 0; i < 2 && e == cudaSuccess; i++) e = cudaEventCreateWithFlags(&s->ds_ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      if (s->stream) cudaStreamDestroy(s->stream);
      if (s->pinned) cudaFreeHost(s->pinned);
      delete s;
      return set_error(PAI_ERR_CUDA, "checkpoint I/O setup failed: %s", cudaGetErrorString(e));
    }
    ctx->io = s;
  }
  *out = ctx->io;
  return PAI_OK;
}

// ---------------------------------------------------------------- byte helpers (little-endian host)
static void put_bytes(std::vector<uint8_t>& b, const void* p, size_t n) {
  const uint8_t* c = static_cast<const uint8_t*>(p);
  b.insert(b.end(), c, c + n);
}
template <typename T>
static void put(std::vector<uint8_t>& b, T v) { put_bytes(b, &v, sizeof v); }

// One payload, device -> file: chunk k crosses to pinned memory on `stream` while chunk k-1 is written.
static bool stream_to_file(IoState* io, FILE* f, const float* dptr, int64_t count, cudaStream_t stream, std::string* err) {
  const size_t bytes = (size_t)count * 4;
  const size_t nch = (bytes + kIoChunk - 1) / kIoChunk;
  const char* src = reinterpret_cast<const char*>(dptr);
  for (size_t k = 0; k <= nch; k++) {
    if (k < nch) {
      const size_t len = std::min(kIoChunk, bytes - k * kIoChunk);
      cudaError_t e = cudaMemcpyAsync(io->pinned + (k & 1) * kIoChunk, src + k * kIoChunk, len, cudaMemcpyDeviceToHost, stream);
      if (e == cudaSuccess) e = cudaEventRecord(io->ev[k & 1], stream);
      if (e != cudaSuccess) { *err = std::string("checkpoint copy to host failed: ") + cudaGetErrorString(e); return false; }
    }
    if (k >= 1) {
      const size_t j = k - 1, len = std::min(kIoChunk, bytes - j * kIoChunk);
      cudaError_t e = cudaEventSynchronize(io->ev[j & 1]);
      if (e != cudaSuccess) { *err = std::string("checkpoint copy to host failed: ") + cudaGetErrorString(e); return false; }
      if (fwrite(io->pinned + (j & 1) * kIoChunk, 1, len, f) != len) {
        *err = std::string("checkpoint write failed: ") + strerror(errno);
        return false;
      }
    }
  }
  return true;
}

// What the writer needs: the file, each tensor's header bytes and its dense device source.
struct SaveJob {
  FILE* f = nullptr;
  std::string path;
  std::vector<uint8_t> head;                   // magic .. tensorCount
  std::vector<std::vector<uint8_t>> theads;    // per tensor: nameLen .. byteLen
  std::vector<const float*> src;
  std::vector<int64_t> count;
};

static bool write_job(IoState* io, const SaveJob& job, cudaStream_t stream, std::string* err) {
  if (fwrite(job.head.data(), 1, job.head.size(), job.f) != job.head.size()) {
    *err = std::string("checkpoint write failed: ") + strerror(errno);
    return false;
  }
  for (size_t i = 0; i < job.theads.size(); i++) {
    if (fwrite(job.theads[i].data(), 1, job.theads[i].size(), job.f) != job.theads[i].size()) {
      *err = std::string("checkpoint write failed: ") + strerror(errno);
      return false;
    }
    if (job.count[i] > 0 && !stream_to_file(io, job.f, job.src[i], job.count[i], stream, err)) return false;
  }
  return true;
}

// Joins a save in flight and releases its snapshot; returns the writer's status (message set on this thread).
static pai_status join_save(pai_ctx* ctx) {
  IoState* io = ctx->io;
  if (!io || !io->writing) return PAI_OK;
  io->writer.join();
  io->writing = false;
  if (io->snapshot) {
    raw_free(ctx, io->snapshot);
    io->snapshot = nullptr;
  }
  pai_status st = io->save_status;
  io->save_status = PAI_OK;
  if (st != PAI_OK) return set_error(st, "%s", io->save_error.c_str());
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

void pai_io_destroy(pai_ctx* ctx) {
  IoState* io = ctx->io;
  if (!io) return;
  if (io->writing) {
    io->writer.join();
    io->writing = false;
  }
  if (io->map) munmap(const_cast<uint8_t*>(io->map), io->map_bytes);
  if (io->fd >= 0) close(io->fd);
  for (int i = 0; i < 2; i++) {
    if (io->ds_pinned[i]) cudaFreeHost(io->ds_pinned[i]);
    cudaEventDestroy(io->ds_ev[i]);
    cudaEventDestroy(io->ev[i]);
  }
  cudaEventDestroy(io->mark);
  cudaFreeHost(io->pinned);
  cudaStreamDestroy(io->stream);
  delete io;
  ctx->io = nullptr;
}

// ---------------------------------------------------------------- checkpoint save
PAI_API pai_status pai_ckpt_save(pai_ctx* ctx, const char* path, int32_t step, const char* metadata, int64_t meta_len,
                                 const char* names, int64_t names_len, const pai_tensor* tensors, int32_t n_tensors) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(join_save(ctx));  // one save in flight per context: the previous one finishes (and reports) first
  if (!path || n_tensors < 0 || (n_tensors > 0 && (!tensors || !names)) || meta_len < 0 || (meta_len > 0 && !metadata))
    return set_error(PAI_ERR_ARGUMENT, "SaveCheckpoint: bad arguments");
  if (meta_len > INT32_MAX) return set_error(PAI_ERR_ARGUMENT, "SaveCheckpoint: metadata of %lld bytes", (long long)meta_len);
  if (ctx->capture) return set_error(PAI_ERR_INVALID_OP, "a checkpoint cannot be saved inside a captured graph");
  IoState* io;
  PAI_TRY(io_state(ctx, &io));

  // Names: n_tensors NUL-terminated strings packed into names[0, names_len).
  SaveJob job;
  job.path = path;
  std::vector<std::string> nm;
  for (int64_t p = 0; (int32_t)nm.size() < n_tensors;) {
    const void* z = p < names_len ? memchr(names + p, 0, (size_t)(names_len - p)) : nullptr;
    if (!z) return set_error(PAI_ERR_ARGUMENT, "SaveCheckpoint: %d names expected in %lld bytes", n_tensors, (long long)names_len);
    const int64_t e = static_cast<const char*>(z) - names;
    nm.emplace_back(names + p, (size_t)(e - p));
    p = e + 1;
  }
  int64_t total = 0;
  for (int32_t i = 0; i < n_tensors; i++) {
    PAI_TRY(check_view(ctx, &tensors[i], "tensor"));
    if (tensors[i].dtype != PAI_F32)  // Checkpoint.cs:39-40 (this backend holds F32 tensors only)
      return set_error(PAI_ERR_UNSUPPORTED, "checkpoint stores float weights; tensor '%s' is not F32.", nm[(size_t)i].c_str());
    const int64_t n = numel(tensors[i]);
    if (n > INT32_MAX)  // Checkpoint.cs:41-42
      return set_error(PAI_ERR_UNSUPPORTED, "tensor '%s' has %lld elements, exceeding this format's 2^31 limit.",
                       nm[(size_t)i].c_str(), (long long)n);
    total += n;
  }

  // Header bytes (Checkpoint.cs:30-35, 44-52).
  put_bytes(job.head, "PAICKPT2", 8);
  put<int32_t>(job.head, step);
  put<int32_t>(job.head, (int32_t)meta_len);
  if (meta_len > 0) put_bytes(job.head, metadata, (size_t)meta_len);
  put<int32_t>(job.head, n_tensors);
  for (int32_t i = 0; i < n_tensors; i++) {
    std::vector<uint8_t> h;
    put<int32_t>(h, (int32_t)nm[(size_t)i].size());
    put_bytes(h, nm[(size_t)i].data(), nm[(size_t)i].size());
    put<int32_t>(h, tensors[i].rank);
    for (int d = 0; d < tensors[i].rank; d++) put<int32_t>(h, tensors[i].dims[d]);
    put<int64_t>(h, numel(tensors[i]) * 4);
    job.theads.push_back(std::move(h));
    job.count.push_back(numel(tensors[i]));
  }
  job.f = fopen(path, "wb");
  if (!job.f) return set_error(PAI_ERR_IO, "could not create '%s': %s", path, strerror(errno));

  // The snapshot: every tensor densely, back to back, on the compute stream.
  void* snap = nullptr;
  pai_status st = total > 0 ? raw_alloc(ctx, (size_t)total * 4, &snap) : PAI_OK;
  if (st == PAI_OK && snap) {
    float* dst = static_cast<float*>(snap);
    for (int32_t i = 0; i < n_tensors; i++) {
      job.src.push_back(dst);
      if (job.count[(size_t)i] > 0) {
        st = gather_dense(ctx, tensors[i], dst);
        if (st != PAI_OK) break;
      }
      dst += job.count[(size_t)i];
    }
  }
  if (st != PAI_OK || (total > 0 && !snap)) {
    // No room for a snapshot: stream from the tensors themselves (dense copies one at a time), caller waiting.
    if (snap) raw_free(ctx, snap);
    std::string err;
    bool ok = fwrite(job.head.data(), 1, job.head.size(), job.f) == job.head.size();
    if (!ok) err = std::string("checkpoint write failed: ") + strerror(errno);
    for (int32_t i = 0; ok && i < n_tensors; i++) {
      ok = fwrite(job.theads[(size_t)i].data(), 1, job.theads[(size_t)i].size(), job.f) == job.theads[(size_t)i].size();
      if (!ok) { err = std::string("checkpoint write failed: ") + strerror(errno); break; }
      if (job.count[(size_t)i] == 0) continue;
      const float* d = nullptr;
      Scratch hold;
      pai_status s2 = dense_input(ctx, tensors[i], &d, &hold);
      if (s2 != PAI_OK) { fclose(job.f); return s2; }
      PAI_CUDA(cudaEventRecord(io->mark, ctx->stream));
      PAI_CUDA(cudaStreamWaitEvent(io->stream, io->mark, 0));
      ok = stream_to_file(io, job.f, d, job.count[(size_t)i], io->stream, &err);
    }
    if (fclose(job.f) != 0 && ok) { ok = false; err = std::string("checkpoint write failed: ") + strerror(errno); }
    if (!ok) return set_error(PAI_ERR_IO, "%s", err.c_str());
    return PAI_OK;
  }
  PAI_CUDA(cudaEventRecord(io->mark, ctx->stream));
  PAI_CUDA(cudaStreamWaitEvent(io->stream, io->mark, 0));
  io->snapshot = snap;
  io->writing = true;
  io->save_status = PAI_OK;
  io->save_error.clear();
  const int device = ctx->device;
  io->writer = std::thread([io, device, job = std::move(job)]() mutable {
    cudaSetDevice(device);
    std::string err;
    bool ok = write_job(io, job, io->stream, &err);
    if (fclose(job.f) != 0 && ok) { ok = false; err = std::string("checkpoint write failed: ") + strerror(errno); }
    if (!ok) {
      io->save_status = PAI_ERR_IO;
      io->save_error = "'" + job.path + "': " + err;
    }
  });
  return PAI_OK;
}

PAI_API pai_status pai_ckpt_wait(pai_ctx* ctx) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  return join_save(ctx);
}

// ---------------------------------------------------------------- checkpoint load
namespace {
struct FileCloser {
  FILE* f;
  ~FileCloser() { if (f) fclose(f); }
};

// Reads [pos, pos + len) of the file into buf, split into up to kLoadReaders contiguous parts read concurrently (one
// on the calling thread): a single reader copying out of the page cache holds a load to ~2 GB/s. Returns the bytes
// read from the start of the range up to the first short part, i.e. up to the end of the file.
constexpr int kLoadReaders = 4;
size_t pread_parts(int fd, char* buf, size_t len, int64_t pos) {
  const size_t min_part = size_t(4) << 20;
  int parts = (int)std::min<size_t>((size_t)kLoadReaders, std::max<size_t>(1, (len + min_part - 1) / min_part));
  const size_t part = (((len + parts - 1) / parts) + 4095) & ~size_t(4095);
  size_t got[kLoadReaders] = {};
  auto work = [&](int i) {
    const size_t b = (size_t)i * part, e = std::min(len, b + part);
    size_t n = 0;
    while (b + n < e) {
      ssize_t r = pread(fd, buf + b + n, e - b - n, (off_t)(pos + (int64_t)(b + n)));
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) break;
      n += (size_t)r;
    }
    got[i] = n;
  };
  std::thread th[kLoadReaders];
  int started = 0;
  for (int i = 1; i < parts && (size_t)i * part < len; i++) {
    try {
      th[started] = std::thread(work, i);
      started++;
    } catch (...) {  // no thread to be had: this part is read here (entry points never throw)
      work(i);
    }
  }
  work(0);
  for (int i = 0; i < started; i++) th[i].join();
  size_t total = 0;
  for (int i = 0; i < parts && (size_t)i * part < len; i++) {
    const size_t want = std::min(len, (size_t)i * part + part) - (size_t)i * part;
    total += got[i];
    if (got[i] < want) break;
  }
  return total;
}
}  // namespace

// Reads the file's header (and, unless header_only, every tensor onto the device, allocated in the current scope);
// pai_ckpt_meta / pai_ckpt_tensor return them. The checks and messages follow Checkpoint.cs:59-139.
PAI_API pai_status pai_ckpt_load(pai_ctx* ctx, const char* path, int32_t header_only, int32_t* step, int64_t* meta_len,
                                 int32_t* n_tensors) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  if (!path) return set_error(PAI_ERR_ARGUMENT, "LoadCheckpoint: bad arguments");
  if (ctx->capture) return set_error(PAI_ERR_INVALID_OP, "a checkpoint cannot be loaded inside a captured graph");
  IoState* io;
  PAI_TRY(io_state(ctx, &io));
  io->meta.clear();
  io->names.clear();
  io->tensors.clear();
  FileCloser fc{fopen(path, "rb")};
  if (!fc.f) return set_error(PAI_ERR_IO, "could not open '%s': %s", path, strerror(errno));
  FILE* f = fc.f;
  auto rd = [&](void* p, size_t n) { return fread(p, 1, n, f); };
  char magic[8];
  if (rd(magic, 8) != 8 || memcmp(magic, "PAICKPT2", 8) != 0)
    return set_error(PAI_ERR_INVALID_DATA, "'%s' is not a ProjectAI checkpoint (bad magic).", path);
  auto rd32 = [&](int32_t* v, const char* what) -> pai_status {
    if (rd(v, 4) != 4) return set_error(PAI_ERR_INVALID_DATA, "'%s' is truncated reading %s.", path, what);
    return PAI_OK;
  };
  int32_t stp = 0, mlen = 0, count = 0;
  PAI_TRY(rd32(&stp, "the step"));
  PAI_TRY(rd32(&mlen, "the metadata length"));
  if (mlen < 0 || mlen > kMaxMeta) return set_error(PAI_ERR_INVALID_DATA, "'%s' has a bad metadata length (%d).", path, mlen);
  io->meta.resize((size_t)mlen);
  size_t got = mlen > 0 ? rd(&io->meta[0], (size_t)mlen) : 0;
  if (got != (size_t)mlen)
    return set_error(PAI_ERR_INVALID_DATA, "'%s' is truncated reading metadata (expected %d bytes, got %zu).", path, mlen, got);
  if (step) *step = stp;
  if (meta_len) *meta_len = mlen;
  if (n_tensors) *n_tensors = 0;
  if (header_only) return PAI_OK;
  PAI_TRY(rd32(&count, "the tensor count"));
  if (count < 0) return set_error(PAI_ERR_INVALID_DATA, "'%s' has a negative tensor count (%d).", path, count);

  std::vector<pai_tensor> loaded;
  auto fail = [&](pai_status st) {  // drop what was allocated, once its copies are done
    cudaStreamSynchronize(io->stream);
    for (auto& t : loaded) pai_release(ctx, t.base);
    io->names.clear();
    io->tensors.clear();
    return st;
  };
  size_t chunk = 0;  // running pinned-buffer counter across tensors
  for (int32_t i = 0; i < count; i++) {
    int32_t nlen = 0, rank = 0;
    pai_status st = rd32(&nlen, "a tensor name length");
    if (st != PAI_OK) return fail(st);
    if (nlen < 0 || nlen > kMaxName)
      return fail(set_error(PAI_ERR_INVALID_DATA, "'%s' tensor %d: bad name length %d.", path, i, nlen));
    std::string name((size_t)nlen, '\0');
    got = nlen > 0 ? rd(&name[0], (size_t)nlen) : 0;
    if (got != (size_t)nlen)
      return fail(set_error(PAI_ERR_INVALID_DATA, "'%s' is truncated reading tensor %d name (expected %d bytes, got %zu).",
                            path, i, nlen, got));
    if ((st = rd32(&rank, "a tensor rank")) != PAI_OK) return fail(st);
    if (rank < 0 || rank > PAI_MAX_RANK)
      return fail(set_error(PAI_ERR_INVALID_DATA, "checkpoint tensor '%s' has invalid rank %d.", name.c_str(), rank));
    int32_t dims[PAI_MAX_RANK] = {};
    int64_t expected = 4;
    bool overflow = false;
    for (int d = 0; d < rank; d++) {
      if ((st = rd32(&dims[d], "a tensor dimension")) != PAI_OK) return fail(st);
      if (dims[d] < 0)
        return fail(set_error(PAI_ERR_INVALID_DATA, "checkpoint tensor '%s' has a negative dimension %d.", name.c_str(), dims[d]));
      if (dims[d] > 0 && expected > INT64_MAX / dims[d]) overflow = true;
      else expected *= dims[d];
    }
    int64_t blen = 0;
    if (rd(&blen, 8) != 8) return fail(set_error(PAI_ERR_INVALID_DATA, "'%s' is truncated reading a payload length.", path));
    if (overflow || blen != expected || blen > INT32_MAX)
      return fail(set_error(PAI_ERR_INVALID_DATA, "checkpoint tensor '%s': payload length %lld != dims product × 4 (%lld).",
                            name.c_str(), (long long)blen, (long long)expected));
    pai_tensor t;
    if ((st = alloc_tensor(ctx, rank, dims, PAI_F32, false, &t)) != PAI_OK) return fail(st);
    loaded.push_back(t);
    // The block may have been freed by work still queued on the compute stream: the copies start after it.
    if (cudaEventRecord(io->mark, ctx->stream) != cudaSuccess || cudaStreamWaitEvent(io->stream, io->mark, 0) != cudaSuccess)
      return fail(set_error(PAI_ERR_CUDA, "checkpoint load: stream ordering failed"));
    char* dst = static_cast<char*>(t.base);
    const int64_t pos = (int64_t)ftello(f);  // the payload's file offset (stdio's buffered position)
    for (int64_t off = 0; off < blen; off += (int64_t)kIoChunk, chunk++) {
      const size_t len = (size_t)std::min<int64_t>((int64_t)kIoChunk, blen - off);
      char* buf = io->pinned + (chunk & 1) * kIoChunk;
      cudaEventSynchronize(io->ev[chunk & 1]);  // the copy that last read this buffer is done
      got = pread_parts(fileno(f), buf, len, pos + off);
      if (got != len)
        return fail(set_error(PAI_ERR_INVALID_DATA, "'%s' is truncated reading tensor '%s' payload (expected %lld bytes, got %lld).",
                              path, name.c_str(), (long long)blen, (long long)(off + (int64_t)got)));
      if (cudaMemcpyAsync(dst + off, buf, len, cudaMemcpyHostToDevice, io->stream) != cudaSuccess ||
          cudaEventRecord(io->ev[chunk & 1], io->stream) != cudaSuccess)
        return fail(set_error(PAI_ERR_CUDA, "checkpoint load: copy to the device failed"));
    }
    if (blen > 0 && fseeko(f, (off_t)(pos + blen), SEEK_SET) != 0)  // stdio resumes after the payload
      return fail(set_error(PAI_ERR_IO, "could not seek in '%s': %s", path, strerror(errno)));
    io->names.push_back(std::move(name));
    io->tensors.push_back(t);
  }
  // Later work on the compute stream sees the loaded tensors.
  PAI_CUDA(cudaEventRecord(io->mark, io->stream));
  PAI_CUDA(cudaStreamWaitEvent(ctx->stream, io->mark, 0));
  if (n_tensors) *n_tensors = count;
  return PAI_OK;
}

PAI_API pai_status pai_ckpt_meta(pai_ctx* ctx, char* buf, int64_t cap) {
  if (!ctx || !ctx->io || (!buf && cap > 0)) return set_error(PAI_ERR_ARGUMENT, "no checkpoint loaded");
  if (cap < (int64_t)ctx->io->meta.size())
    return set_error(PAI_ERR_ARGUMENT, "metadata needs %zu bytes, buffer holds %lld", ctx->io->meta.size(), (long long)cap);
  if (!ctx->io->meta.empty()) memcpy(buf, ctx->io->meta.data(), ctx->io->meta.size());
  return PAI_OK;
}

PAI_API pai_status pai_ckpt_tensor(pai_ctx* ctx, int32_t index, char* name, int64_t name_cap, int64_t* name_len,
                                   pai_tensor* out) {
  if (!ctx || !ctx->io) return set_error(PAI_ERR_ARGUMENT, "no checkpoint loaded");
  IoState* io = ctx->io;
  if (index < 0 || index >= (int32_t)io->tensors.size())
    return set_error(PAI_ERR_OUT_OF_RANGE, "checkpoint tensor index %d out of range [0, %zu)", index, io->tensors.size());
  const std::string& n = io->names[(size_t)index];
  if (name_len) *name_len = (int64_t)n.size();
  if (name) {
    if (name_cap < (int64_t)n.size()) return set_error(PAI_ERR_ARGUMENT, "name needs %zu bytes", n.size());
    if (!n.empty()) memcpy(name, n.data(), n.size());
  }
  if (out) *out = io->tensors[(size_t)index];
  return PAI_OK;
}

PAI_API pai_status pai_ckpt_close(pai_ctx* ctx) {
  if (ctx && ctx->io) {
    ctx->io->meta.clear();
    ctx->io->names.clear();
    ctx->io->tensors.clear();
  }
  return PAI_OK;
}

// ---------------------------------------------------------------- packed token datasets
namespace pai {
// inputs[r][t] = ids[r][t], targets[r][t] = ids[r][t + 1] for each block r of seq + 1 ids (Training.cs:127-136), as
// F32 ids (the convention of Embedding.cs:38-45 and Loss.cs:26-33): int -> float rounds to nearest, as C# does.
template <typename T>
__global__ void k_widen_ids(const T* __restrict__ raw, int64_t rows, int seq, float* __restrict__ in,
                            float* __restrict__ tg) {
  const int64_t n = rows * seq;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / seq, t = i - r * seq;
    const T* blk = raw + r * (int64_t)(seq + 1);
    in[i] = (float)(int32_t)blk[t];
    tg[i] = (float)(int32_t)blk[t + 1];
  }
}
}  // namespace pai

// Maps the shard of a packed dataset: block_count blocks of seq_len + 1 little-endian ids, elem_bytes (2 = "u16",
// 4 = "u32") each (PackedBinDataset.cs:43-95). Replaces the context's open dataset.
PAI_API pai_status pai_dataset_open(pai_ctx* ctx, const char* bin_path, int32_t elem_bytes, int32_t seq_len,
                                    int64_t block_count) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  if (!bin_path) return set_error(PAI_ERR_ARGUMENT, "OpenDataset: bad arguments");
  if (elem_bytes != 2 && elem_bytes != 4)
    return set_error(PAI_ERR_INVALID_DATA, "unsupported dataset dtype (%d-byte ids).", elem_bytes);
  if (seq_len < 1) return set_error(PAI_ERR_INVALID_DATA, "manifest SequenceLength must be >= 1; got %d.", seq_len);
  if (block_count < 1) return set_error(PAI_ERR_INVALID_DATA, "manifest BlockCount must be >= 1; got %lld.", (long long)block_count);
  if (block_count > INT32_MAX)  // PackedBinDataset.cs:35: Count = checked((int)BlockCount)
    return set_error(PAI_ERR_INVALID_DATA, "manifest BlockCount %lld exceeds the dataset's int32 count.", (long long)block_count);
  IoState* io;
  PAI_TRY(io_state(ctx, &io));
  const int blk = seq_len + 1;
  const int64_t needed = block_count * blk * elem_bytes;
  const int fd = open(bin_path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return set_error(PAI_ERR_IO, "dataset shard '%s' (from manifest) not found: %s", bin_path, strerror(errno));
  struct stat sb;
  if (fstat(fd, &sb) != 0) {
    close(fd);
    return set_error(PAI_ERR_IO, "dataset shard '%s': %s", bin_path, strerror(errno));
  }
  if ((int64_t)sb.st_size < needed) {
    close(fd);
    return set_error(PAI_ERR_INVALID_DATA,
                     "dataset shard '%s' is %lld bytes but the manifest needs %lld for %lld blocks of %d %s ids.", bin_path,
                     (long long)sb.st_size, (long long)needed, (long long)block_count, blk, elem_bytes == 2 ? "u16" : "u32");
  }
  void* m = mmap(nullptr, (size_t)needed, PROT_READ, MAP_SHARED, fd, 0);
  if (m == MAP_FAILED) {
    close(fd);
    return set_error(PAI_ERR_IO, "dataset shard '%s': mmap failed: %s", bin_path, strerror(errno));
  }
  if (io->map) munmap(const_cast<uint8_t*>(io->map), io->map_bytes);
  if (io->fd >= 0) close(io->fd);
  io->fd = fd;
  io->map = static_cast<const uint8_t*>(m);
  io->map_bytes = (size_t)needed;
  io->elem = elem_bytes;
  io->seq = seq_len;
  io->blocks = block_count;
  return PAI_OK;
}

// One micro-batch: blocks indices[0, count) of the open dataset as device F32 ids, inputs and targets [count, seq_len]
// (ids[:, :-1] and ids[:, 1:] of each block, Training.cs:122-141), allocated in the current scope.
PAI_API pai_status pai_dataset_batch(pai_ctx* ctx, const int64_t* indices, int32_t count, pai_tensor* inputs,
                                     pai_tensor* targets) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  IoState* io = ctx->io;
  if (!io || !io->map) return set_error(PAI_ERR_INVALID_OP, "no dataset is open");
  if (count < 1 || !indices || !inputs || !targets) return set_error(PAI_ERR_ARGUMENT, "NextBatch: bad arguments");
  if (ctx->capture) return set_error(PAI_ERR_INVALID_OP, "a host upload cannot be part of a captured graph");
  for (int32_t r = 0; r < count; r++)
    if (indices[r] < 0 || indices[r] >= io->blocks)  // PackedBinDataset.cs:98-99
      return set_error(PAI_ERR_OUT_OF_RANGE, "index %lld: valid range is [0, %lld).", (long long)indices[r], (long long)io->blocks);
  const size_t blk_bytes = (size_t)(io->seq + 1) * io->elem;
  const size_t bytes = blk_bytes * (size_t)count;
  // Two pinned buffers, each reused once the upload that last read it is done.
  const int b = io->ds_next;
  io->ds_next ^= 1;
  PAI_CUDA(cudaEventSynchronize(io->ds_ev[b]));
  if (bytes > io->ds_cap) {
    for (int i = 0; i < 2; i++) {
      PAI_CUDA(cudaEventSynchronize(io->ds_ev[i]));
      if (io->ds_pinned[i]) cudaFreeHost(io->ds_pinned[i]);
      io->ds_pinned[i] = nullptr;
    }
    io->ds_cap = 0;
    for (int i = 0; i < 2; i++)
      PAI_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&io->ds_pinned[i]), bytes, cudaHostAllocDefault));
    io->ds_cap = bytes;
  }
  char* stage = io->ds_pinned[b];
  for (int32_t r = 0; r < count; r++) memcpy(stage + (size_t)r * blk_bytes, io->map + (size_t)indices[r] * blk_bytes, blk_bytes);
  if (io->elem == 4) {  // GetSequence's checked((int)raw[i]) (PackedBinDataset.cs:110)
    const uint32_t* ids = reinterpret_cast<const uint32_t*>(stage);
    for (size_t i = 0; i < bytes / 4; i++)
      if (ids[i] > (uint32_t)INT32_MAX)
        return set_error(PAI_ERR_OUT_OF_RANGE, "id %u in block %lld exceeds the int32 range.", ids[i],
                         (long long)indices[i / (size_t)(io->seq + 1)]);
  }
  Scratch raw;
  PAI_TRY(scratch(ctx, bytes, &raw));
  PAI_CUDA(cudaMemcpyAsync(raw.p, stage, bytes, cudaMemcpyHostToDevice, ctx->stream));
  PAI_CUDA(cudaEventRecord(io->ds_ev[b], ctx->stream));
  const int32_t dims[2] = {count, io->seq};
  pai_tensor in, tg;
  PAI_TRY(alloc_tensor(ctx, 2, dims, PAI_F32, false, &in));
  pai_status st = alloc_tensor(ctx, 2, dims, PAI_F32, false, &tg);
  if (st != PAI_OK) {
    pai_release(ctx, in.base);
    return st;
  }
  const int64_t n = (int64_t)count * io->seq;
  if (io->elem == 2)
    k_widen_ids<uint16_t><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(static_cast<const uint16_t*>(raw.p), count, io->seq,
                                                                           fptr(in), fptr(tg));
  else
    k_widen_ids<uint32_t><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(static_cast<const uint32_t*>(raw.p), count, io->seq,
                                                                           fptr(in), fptr(tg));
  PAI_LAUNCH_CHECK("dataset ids");
  *inputs = in;
  *targets = tg;
  return PAI_OK;
}

PAI_API pai_status pai_dataset_close(pai_ctx* ctx) {
  if (!ctx) return PAI_OK;
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  IoState* io = ctx->io;
  if (!io) return PAI_OK;
  for (int i = 0; i < 2; i++) cudaEventSynchronize(io->ds_ev[i]);
  if (io->map) munmap(const_cast<uint8_t*>(io->map), io->map_bytes);
  if (io->fd >= 0) close(io->fd);
  io->map = nullptr;
  io->map_bytes = 0;
  io->fd = -1;
  io->blocks = 0;
  return PAI_OK;
}
