// Context, caching allocator, scopes, host transfer and strided copy.
// Contract: ProjectAI.Core/IComputeBackend.cs:14-18 (Allocate/FromHost/ToHost/Copy) and :69-95 (scopes), with
// the lifetime semantics of ProjectAI.Backends.Torch/TorchComputeBackend.cs:208-218.
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"

namespace pai {

static thread_local std::string t_error;

pai_status set_error(pai_status st, const char* fmt, ...) {
  char buf[2048];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_error = buf;
  return st;
}

pai_status cuda_error(cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation)
    return set_error(PAI_ERR_OUT_OF_MEMORY, "CUDA out of memory (%s): %s", what, cudaGetErrorString(e));
  return set_error(PAI_ERR_CUDA, "CUDA error in %s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}


pai_status enter(pai_ctx* ctx) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != ctx->device) PAI_CUDA(cudaSetDevice(ctx->device));
  return PAI_OK;
}

// Size classes: 512-byte granularity below 1 MiB, 2 MiB above. A training step allocates the same sizes every
// step, so after the first step every request is a cache hit.
static size_t round_size(size_t bytes) {
  if (bytes == 0) bytes = 1;
  if (bytes < (1u << 20)) return (bytes + 511) & ~size_t(511);
  return (bytes + (size_t(2) << 20) - 1) & ~((size_t(2) << 20) - 1);
}

static void release_cache(pai_ctx* ctx) {
  cudaStreamSynchronize(ctx->stream);
  for (auto& kv : ctx->free_blocks) {
    for (void* p : kv.second) { cudaFree(p); ctx->reserved -= (int64_t)kv.first; }
  }
  ctx->free_blocks.clear();
}

pai_status raw_alloc(pai_ctx* ctx, size_t bytes, void** out) {
  size_t sz = round_size(bytes);
  if (ctx->capture) {
    // inside a capture: reuse a block this graph already owns, else take one and make the graph its owner
    auto pit = ctx->capture->pool.parked.find(sz);
    if (pit != ctx->capture->pool.parked.end() && !pit->second.empty()) {
      *out = pit->second.back();
      pit->second.pop_back();
      ctx->live[*out] = BlockInfo{sz, -1};
      ctx->in_use += (int64_t)sz;
      if (ctx->in_use > ctx->peak) ctx->peak = ctx->in_use;
      return PAI_OK;
    }
  }
  auto it = ctx->free_blocks.find(sz);
  if (it != ctx->free_blocks.end() && !it->second.empty()) {
    *out = it->second.back();
    it->second.pop_back();
  } else {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, sz);
    if (e != cudaSuccess) {
      cudaGetLastError();
      release_cache(ctx);  // give cached blocks back to the driver and retry once
      e = cudaMalloc(&p, sz);
      if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(PAI_ERR_OUT_OF_MEMORY,
                         "CUDA out of memory: failed to allocate %zu bytes on device %d (in use %lld, reserved %lld)",
                         sz, ctx->device, (long long)ctx->in_use, (long long)ctx->reserved);
      }
    }
    ctx->reserved += (int64_t)sz;
    *out = p;
  }
  ctx->live[*out] = BlockInfo{sz, -1};
  ctx->in_use += (int64_t)sz;
  if (ctx->in_use > ctx->peak) ctx->peak = ctx->in_use;
  if (ctx->capture) {
    ctx->capture->pool.owned.insert(*out);
    ctx->graph_owner[*out] = ctx->capture;
  }
  return PAI_OK;
}

void raw_free(pai_ctx* ctx, void* p) {
  auto it = ctx->live.find(p);
  if (it == ctx->live.end()) return;
  size_t sz = it->second.bytes;
  ctx->in_use -= (int64_t)sz;
  ctx->live.erase(it);
  auto own = ctx->graph_owner.find(p);
  if (own != ctx->graph_owner.end()) {
    own->second->pool.parked[sz].push_back(p);  // a graph still reads or writes it: keep it out of the cache
    return;
  }
  ctx->free_blocks[sz].push_back(p);
}

pai_status alloc_tensor(pai_ctx* ctx, int rank, const int32_t* dims, int dtype, bool zero, pai_tensor* out) {
  if (rank < 0 || rank > PAI_MAX_RANK) return set_error(PAI_ERR_ARGUMENT, "rank %d is not supported (max %d)", rank, PAI_MAX_RANK);
  int64_t n = 1;
  for (int i = 0; i < rank; i++) {
    if (dims[i] < 0) return set_error(PAI_ERR_OUT_OF_RANGE, "Dimensions must be non-negative.");
    n *= dims[i];
  }
  void* p = nullptr;
  PAI_TRY(raw_alloc(ctx, (size_t)n * 4, &p));
  if (!ctx->scopes.empty()) {
    ctx->live[p].scope = (int)ctx->scopes.size() - 1;
    ctx->scopes.back().insert(p);
  }
  if (zero && n > 0) PAI_CUDA(cudaMemsetAsync(p, 0, (size_t)n * 4, ctx->stream));
  set_contiguous(out, p, rank, dims, dtype);
  return PAI_OK;
}

pai_status scratch(pai_ctx* ctx, size_t bytes, Scratch* s) {
  s->ctx = ctx;
  return raw_alloc(ctx, bytes, &s->p);
}

pai_status h2d(pai_ctx* ctx, void* dst, const void* host, size_t bytes) {
  if (bytes == 0) return PAI_OK;
  if (ctx->capture)
    return set_error(PAI_ERR_INVALID_OP, "a host upload cannot be part of a captured graph; pass device tensors instead");
  if (bytes > kPinnedChunk) {
    PAI_CUDA(cudaMemcpyAsync(dst, host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return PAI_OK;
  }
  if (!ctx->pinned) {
    PAI_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&ctx->pinned), kPinnedChunk * kPinnedChunks, cudaHostAllocDefault));
    for (int i = 0; i < kPinnedChunks; i++) PAI_CUDA(cudaEventCreateWithFlags(&ctx->pinned_ev[i], cudaEventDisableTiming));
  }
  int c = ctx->pinned_next;
  ctx->pinned_next = (c + 1) % kPinnedChunks;
  PAI_CUDA(cudaEventSynchronize(ctx->pinned_ev[c]));  // the copy that last read this chunk has completed
  char* slot = ctx->pinned + (size_t)c * kPinnedChunk;
  memcpy(slot, host, bytes);
  PAI_CUDA(cudaMemcpyAsync(dst, slot, bytes, cudaMemcpyHostToDevice, ctx->stream));
  PAI_CUDA(cudaEventRecord(ctx->pinned_ev[c], ctx->stream));
  return PAI_OK;
}

pai_status upload(pai_ctx* ctx, const void* host, size_t bytes, Scratch* s) {
  PAI_TRY(scratch(ctx, bytes, s));
  return h2d(ctx, s->p, host, bytes);
}

// ---------------------------------------------------------------- views
int64_t numel(const pai_tensor& t) {
  int64_t n = 1;
  for (int i = 0; i < t.rank; i++) n *= t.dims[i];
  return n;
}

std::string shape_str(const pai_tensor& t) {
  std::string s = "[";
  for (int i = 0; i < t.rank; i++) {
    if (i) s += ", ";
    s += std::to_string(t.dims[i]);
  }
  return s + "]";
}

bool is_dense(const pai_tensor& t) {
  int64_t acc = 1;
  for (int i = t.rank - 1; i >= 0; i--) {
    if (t.dims[i] == 1) continue;
    if (t.strides[i] != acc) return false;
    acc *= t.dims[i];
  }
  return true;
}

void set_contiguous(pai_tensor* t, void* base, int rank, const int32_t* dims, int dtype) {
  memset(t, 0, sizeof *t);
  t->base = base;
  t->rank = rank;
  t->dtype = dtype;
  int64_t acc = 1;
  for (int i = rank - 1; i >= 0; i--) {
    t->dims[i] = dims[i];
    t->strides[i] = acc;
    acc *= dims[i];
  }
}

pai_status check_view(pai_ctx* ctx, const pai_tensor* t, const char* what) {
  if (!t) return set_error(PAI_ERR_ARGUMENT, "%s: null tensor", what);
  if (t->rank < 0 || t->rank > PAI_MAX_RANK) return set_error(PAI_ERR_ARGUMENT, "%s: rank %d unsupported", what, t->rank);
  if (t->dtype != PAI_F32) return set_error(PAI_ERR_UNSUPPORTED, "%s: only F32 tensors are supported on this backend", what);
  auto it = ctx->live.find(t->base);
  if (it == ctx->live.end())
    return set_error(PAI_ERR_INVALID_OP, "%s: tensor storage is not a live allocation of this backend (used after its scope ended?)", what);
  int64_t lo = t->offset, hi = t->offset;
  for (int i = 0; i < t->rank; i++) {
    if (t->dims[i] < 0) return set_error(PAI_ERR_ARGUMENT, "%s: negative dimension", what);
    if (t->dims[i] == 0) return PAI_OK;
    int64_t span = (int64_t)(t->dims[i] - 1) * t->strides[i];
    if (span < 0) lo += span; else hi += span;
  }
  if (lo < 0 || (hi + 1) * 4 > (int64_t)it->second.bytes)
    return set_error(PAI_ERR_ARGUMENT, "%s: view %s exceeds its storage", what, shape_str(*t).c_str());
  return PAI_OK;
}

bool broadcast_shape(const pai_tensor& a, const pai_tensor& b, int* rank, int32_t* dims) {
  int n = std::max(a.rank, b.rank);
  if (n > PAI_MAX_RANK) return false;
  for (int i = 0; i < n; i++) {
    int da = i < a.rank ? a.dims[a.rank - 1 - i] : 1;
    int db = i < b.rank ? b.dims[b.rank - 1 - i] : 1;
    int d;
    if (da == db) d = da;
    else if (da == 1) d = db;
    else if (db == 1) d = da;
    else return false;
    dims[n - 1 - i] = d;
  }
  *rank = n;
  return true;
}

pai_tensor broadcast_view(const pai_tensor& t, int rank, const int32_t* dims) {
  pai_tensor r = t;
  int lead = rank - t.rank;
  for (int i = 0; i < rank; i++) {
    r.dims[i] = dims[i];
    if (i < lead) { r.strides[i] = 0; continue; }
    r.strides[i] = (t.dims[i - lead] == dims[i]) ? t.strides[i - lead] : 0;
  }
  r.rank = rank;
  return r;
}

void collapse(int rank, const int32_t* dims, const pai_tensor* const* views, int n, DView* out) {
  // Keep axes with extent > 1, then merge axis i into i+1 when every view has stride[i] == stride[i+1]*dim[i+1].
  int32_t kd[PAI_MAX_RANK];
  int64_t ks[4][PAI_MAX_RANK];
  int k = 0;
  for (int i = 0; i < rank; i++) {
    if (dims[i] == 1) continue;
    kd[k] = dims[i];
    for (int v = 0; v < n; v++) ks[v][k] = views[v]->strides[i];
    k++;
  }
  int32_t md[PAI_MAX_RANK];
  int64_t ms[4][PAI_MAX_RANK];
  int m = 0;
  for (int i = 0; i < k; i++) {
    if (m > 0) {
      bool ok = true;
      for (int v = 0; v < n; v++)
        if (ms[v][m - 1] != ks[v][i] * (int64_t)kd[i]) { ok = false; break; }
      if (ok) {
        md[m - 1] *= kd[i];
        for (int v = 0; v < n; v++) ms[v][m - 1] = ks[v][i];
        continue;
      }
    }
    md[m] = kd[i];
    for (int v = 0; v < n; v++) ms[v][m] = ks[v][i];
    m++;
  }
  for (int v = 0; v < n; v++) {
    out[v].offset = views[v]->offset;
    out[v].rank = m;
    for (int i = 0; i < m; i++) { out[v].dims[i] = md[i]; out[v].strides[i] = ms[v][i]; }
  }
}

// ---------------------------------------------------------------- strided copy kernels
__global__ void k_gather(const float* __restrict__ src, pai::DView sv, float* __restrict__ dst, int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (n < (1ll << 31)) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
      dst[i] = src[dview_offset32(sv, (uint32_t)i)];
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
      dst[i] = src[dview_offset(sv, i)];
  }
}

__global__ void k_copy_strided(const float* __restrict__ src, pai::DView sv, float* __restrict__ dst, pai::DView dv,
                               int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    dst[dview_offset(dv, i)] = src[dview_offset(sv, i)];
}

// Unit-stride rows of `len` elements (a permuted view whose last axis stays contiguous, e.g. the [b,s,h,d] view of a
// [b,h,s,d] tensor): one warp per row, the row's offset from one 32-bit coordinate decomposition.
__global__ void k_gather_rows_view(const float* __restrict__ src, pai::DView rv, float* __restrict__ dst, int64_t rows,
                                   int len) {
  int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    int64_t off, o2, o3;
    row_offsets3(rv, rv, rv, (uint32_t)r, off, o2, o3);
    const float* s = src + off;
    float* d = dst + r * len;
    for (int j = lane; j < len; j += 32) d[j] = s[j];
  }
}

// k_gather_rows_view with one thread per 16-byte group: every row start 16-byte aligned and len % 4 == 0.
__global__ void k_gather_rows_view4(const float* __restrict__ src, pai::DView rv, float* __restrict__ dst, int64_t rows,
                                    int len) {
  const int q = len >> 2;
  const int64_t total = rows * q;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / q;
    const int c = (int)(i - r * q) * 4;
    int64_t off, o2, o3;
    row_offsets3(rv, rv, rv, (uint32_t)r, off, o2, o3);
    *reinterpret_cast<float4*>(dst + r * len + c) = *reinterpret_cast<const float4*>(src + off + c);
  }
}

pai_status gather_dense(pai_ctx* ctx, const pai_tensor& src, float* dst) {
  int64_t n = numel(src);
  if (n == 0) return PAI_OK;
  if (is_dense(src)) {
    PAI_CUDA(cudaMemcpyAsync(dst, fptr(src), (size_t)n * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    return PAI_OK;
  }
  const pai_tensor* v[1] = {&src};
  DView dv;
  collapse(src.rank, src.dims, v, 1, &dv);
  dv.offset = 0;
  if (dv.rank >= 2 && dv.strides[dv.rank - 1] == 1 && dv.dims[dv.rank - 1] >= 32 && n < (1ll << 31)) {
    int len = dv.dims[dv.rank - 1];
    DView rv = dv;
    rv.rank = dv.rank - 1;
    int64_t rows = n / len;
    bool vec4 = len % 4 == 0 && (uintptr_t)fptr(src) % 16 == 0 && (uintptr_t)dst % 16 == 0;
    for (int i = 0; i < rv.rank && vec4; i++)
      if (rv.dims[i] > 1 && rv.strides[i] % 4) vec4 = false;
    if (vec4)
      k_gather_rows_view4<<<grid_for(ctx, n / 4, 256), 256, 0, ctx->stream>>>(fptr(src), rv, dst, rows, len);
    else
      k_gather_rows_view<<<grid_for(ctx, rows * 32, 256), 256, 0, ctx->stream>>>(fptr(src), rv, dst, rows, len);
  } else {
    k_gather<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(fptr(src), dv, dst, n);
  }
  PAI_LAUNCH_CHECK("gather");
  return PAI_OK;
}

pai_status dense_input(pai_ctx* ctx, const pai_tensor& t, const float** out, Scratch* holder) {
  if (is_dense(t)) { *out = fptr(t); return PAI_OK; }
  PAI_TRY(scratch(ctx, (size_t)numel(t) * 4, holder));
  PAI_TRY(gather_dense(ctx, t, static_cast<float*>(holder->p)));
  *out = static_cast<const float*>(holder->p);
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

// ================================================================ C ABI
PAI_API const char* pai_last_error(void) { return t_error.c_str(); }

PAI_API pai_status pai_ctx_create(int device, pai_ctx** out) {
  if (!out) return set_error(PAI_ERR_ARGUMENT, "null out");
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return set_error(PAI_ERR_CUDA, "no CUDA device is available (%s)", cudaGetErrorString(e));
  if (device < 0 || device >= count)
    return set_error(PAI_ERR_OUT_OF_RANGE, "device ordinal %d out of range [0,%d)", device, count);
  PAI_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  PAI_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return set_error(PAI_ERR_UNSUPPORTED, "device %d (%s, sm_%d%d) is not a Blackwell sm_100 GPU", device, prop.name,
                     prop.major, prop.minor);
  auto* c = new pai_ctx();
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  snprintf(c->name, sizeof c->name, "cuda:%d (%s)", device, prop.name);
  cudaError_t e1 = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  cudaError_t e2 = cudaStreamCreateWithFlags(&c->comm_stream, cudaStreamNonBlocking);
  cudaError_t e3 = cudaMalloc(&c->d_error_flag, 64);
  if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess) {
    delete c;
    return set_error(PAI_ERR_CUDA, "failed to create streams for device %d", device);
  }
  cudaMemset(c->d_error_flag, 0, 64);
  *out = c;
  return PAI_OK;
}

void pai_dp_destroy(pai_ctx* ctx);  // dp.cu
void pai_io_destroy(pai_ctx* ctx);  // io.cu

PAI_API pai_status pai_ctx_destroy(pai_ctx* ctx) {
  if (!ctx) return PAI_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  cudaStreamSynchronize(ctx->comm_stream);
  pai_dp_destroy(ctx);
  pai_io_destroy(ctx);  // joins a checkpoint writer still running
  for (auto& kv : ctx->live) cudaFree(kv.first);
  for (auto& kv : ctx->free_blocks)
    for (void* p : kv.second) cudaFree(p);
  for (auto& kv : ctx->graph_owner)  // blocks parked by graphs the caller did not destroy
    if (!ctx->live.count(kv.first)) cudaFree(kv.first);
  cudaFree(ctx->d_error_flag);
  if (ctx->pinned) {
    cudaFreeHost(ctx->pinned);
    for (int i = 0; i < pai::kPinnedChunks; i++) cudaEventDestroy(ctx->pinned_ev[i]);
  }
  for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
  for (auto& kv : ctx->timed)
    for (cudaEvent_t e : kv.second.ev) cudaEventDestroy(e);
  if (ctx->timer_start) { cudaEventDestroy(ctx->timer_start); cudaEventDestroy(ctx->timer_stop); }
  cudaStreamDestroy(ctx->stream);
  cudaStreamDestroy(ctx->comm_stream);
  delete ctx;
  return PAI_OK;
}

PAI_API pai_status pai_sync(pai_ctx* ctx) {
  PAI_TRY(enter(ctx));
  PAI_CUDA(cudaStreamSynchronize(ctx->stream));
  return PAI_OK;
}

PAI_API pai_status pai_device_name(pai_ctx* ctx, char* buf, int32_t n) {
  if (!ctx || !buf || n <= 0) return set_error(PAI_ERR_ARGUMENT, "bad arguments");
  snprintf(buf, (size_t)n, "%s", ctx->name);
  return PAI_OK;
}

PAI_API pai_status pai_alloc(pai_ctx* ctx, int32_t rank, const int32_t* dims, int32_t dtype, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (dtype != PAI_F32) return set_error(PAI_ERR_UNSUPPORTED, "only F32 tensors are supported on this backend");
  return alloc_tensor(ctx, rank, dims, dtype, true, out);
}

PAI_API pai_status pai_from_host(pai_ctx* ctx, const float* host, int64_t count, int32_t rank, const int32_t* dims,
                                 int32_t dtype, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (dtype != PAI_F32) return set_error(PAI_ERR_UNSUPPORTED, "only F32 tensors are supported on this backend");
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, rank, dims, dtype, false, &r));
  int64_t n = numel(r);
  if (count < n) {
    pai_release(ctx, r.base);
    return set_error(PAI_ERR_ARGUMENT, "FromHost: %lld values for a tensor of %lld elements", (long long)count, (long long)n);
  }
  PAI_TRY(h2d(ctx, r.base, host, (size_t)n * 4));
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_to_host(pai_ctx* ctx, const pai_tensor* src, float* host, int64_t count) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, src, "source"));
  int64_t n = numel(*src);
  if (count < n) return set_error(PAI_ERR_ARGUMENT, "ToHost: destination holds %lld of %lld elements", (long long)count, (long long)n);
  if (n == 0) return PAI_OK;
  const float* d = nullptr;
  Scratch hold;
  PAI_TRY(dense_input(ctx, *src, &d, &hold));
  PAI_CUDA(cudaMemcpyAsync(host, d, (size_t)n * 4, cudaMemcpyDeviceToHost, ctx->stream));
  PAI_CUDA(cudaStreamSynchronize(ctx->stream));
  return PAI_OK;
}

PAI_API pai_status pai_copy(pai_ctx* ctx, const pai_tensor* src, const pai_tensor* dst) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, src, "source"));
  PAI_TRY(check_view(ctx, dst, "destination"));
  int64_t n = numel(*src);
  if (n != numel(*dst))
    return set_error(PAI_ERR_ARGUMENT, "Copy: element counts differ (%s vs %s)", shape_str(*src).c_str(), shape_str(*dst).c_str());
  if (n == 0) return PAI_OK;
  if (is_dense(*dst) && src->base != dst->base) return gather_dense(ctx, *src, fptr(*dst));
  // Logical order is row-major over each view's own shape: address both through flat indices.
  const pai_tensor* sv[1] = {src};
  const pai_tensor* dvw[1] = {dst};
  DView s, d;
  collapse(src->rank, src->dims, sv, 1, &s);
  collapse(dst->rank, dst->dims, dvw, 1, &d);
  s.offset = 0;
  d.offset = 0;
  // Source and destination may overlap (a copy into a view of the same storage): stage through a dense buffer.
  if (src->base == dst->base) {
    Scratch tmp;
    PAI_TRY(scratch(ctx, (size_t)n * 4, &tmp));
    PAI_TRY(gather_dense(ctx, *src, static_cast<float*>(tmp.p)));
    DView flat{};
    flat.rank = 1; flat.dims[0] = (int32_t)n; flat.strides[0] = 1;
    k_copy_strided<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(static_cast<float*>(tmp.p), flat, fptr(*dst), d, n);
  } else {
    k_copy_strided<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(fptr(*src), s, fptr(*dst), d, n);
  }
  PAI_LAUNCH_CHECK("copy");
  return PAI_OK;
}

PAI_API pai_status pai_scope_begin(pai_ctx* ctx) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  ctx->scopes.emplace_back();
  return PAI_OK;
}

PAI_API pai_status pai_scope_end(pai_ctx* ctx) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (ctx->scopes.empty()) return set_error(PAI_ERR_INVALID_OP, "scope_end without an open scope");
  auto owned = std::move(ctx->scopes.back());
  ctx->scopes.pop_back();
  for (void* p : owned) raw_free(ctx, p);
  return PAI_OK;
}

PAI_API pai_status pai_keep_alive(pai_ctx* ctx, const void* base) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  void* p = const_cast<void*>(base);
  auto it = ctx->live.find(p);
  if (it == ctx->live.end()) return set_error(PAI_ERR_INVALID_OP, "KeepAlive of a tensor this backend does not own");
  int s = it->second.scope;
  if (s < 0) return PAI_OK;
  ctx->scopes[(size_t)s].erase(p);
  it->second.scope = s - 1;  // exactly one level (IComputeBackend.cs:80-87)
  if (s - 1 >= 0) ctx->scopes[(size_t)(s - 1)].insert(p);
  return PAI_OK;
}

PAI_API pai_status pai_release(pai_ctx* ctx, const void* base) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  void* p = const_cast<void*>(base);
  auto it = ctx->live.find(p);
  if (it == ctx->live.end()) return PAI_OK;
  if (it->second.scope >= 0) ctx->scopes[(size_t)it->second.scope].erase(p);
  raw_free(ctx, p);
  return PAI_OK;
}

PAI_API pai_status pai_finalize(pai_ctx* ctx, const void* base) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  void* p = const_cast<void*>(base);
  auto it = ctx->live.find(p);
  if (it == ctx->live.end() || it->second.scope >= 0) return PAI_OK;
  raw_free(ctx, p);
  return PAI_OK;
}

PAI_API pai_status pai_memory_stats(pai_ctx* ctx, int64_t* in_use, int64_t* peak, int64_t* reserved) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (in_use) *in_use = ctx->in_use;
  if (peak) *peak = ctx->peak;
  if (reserved) *reserved = ctx->reserved;
  return PAI_OK;
}

PAI_API pai_status pai_reset_peak(pai_ctx* ctx) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  ctx->peak = ctx->in_use;
  return PAI_OK;
}

// ================================================================ instrumentation
namespace pai {

static cudaEvent_t pooled_event(pai_ctx* ctx) {
  if (!ctx->event_pool.empty()) {
    cudaEvent_t e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

KernelTimerScope::KernelTimerScope(pai_ctx* c, const char* family, double work) : ctx(c) {
  if (!ctx->kernel_timing || ctx->capture) return;  // replays of a captured graph are timed as a whole
  slot = &ctx->timed[family];
  cudaEvent_t e = pooled_event(ctx);
  cudaEventRecord(e, ctx->stream);
  slot->ev.push_back(e);
  slot->work += work;
  slot->launches++;
}

KernelTimerScope::~KernelTimerScope() {
  if (!slot) return;
  cudaEvent_t e = pooled_event(ctx);
  cudaEventRecord(e, ctx->stream);
  slot->ev.push_back(e);
}

}  // namespace pai

// Stream timer: events recorded on the compute stream itself (the stream every op is ordered on).
PAI_API pai_status pai_timer_start(pai_ctx* ctx) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (!ctx->timer_start) {
    PAI_CUDA(cudaEventCreate(&ctx->timer_start));
    PAI_CUDA(cudaEventCreate(&ctx->timer_stop));
  }
  PAI_CUDA(cudaEventRecord(ctx->timer_start, ctx->stream));
  return PAI_OK;
}

PAI_API pai_status pai_timer_stop(pai_ctx* ctx, float* ms) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (!ctx->timer_start) return set_error(PAI_ERR_INVALID_OP, "timer_stop without timer_start");
  PAI_CUDA(cudaEventRecord(ctx->timer_stop, ctx->stream));
  PAI_CUDA(cudaEventSynchronize(ctx->timer_stop));
  PAI_CUDA(cudaEventElapsedTime(ms, ctx->timer_start, ctx->timer_stop));
  return PAI_OK;
}

PAI_API pai_status pai_launch_count(pai_ctx* ctx, int64_t* n) {
  if (!ctx || !n) return set_error(PAI_ERR_ARGUMENT, "bad arguments");
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  *n = ctx->launches;
  return PAI_OK;
}

PAI_API pai_status pai_kernel_timing(pai_ctx* ctx, int32_t enable) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_CUDA(cudaStreamSynchronize(ctx->stream));
  for (auto& kv : ctx->timed)
    for (cudaEvent_t e : kv.second.ev) ctx->event_pool.push_back(e);
  ctx->timed.clear();
  ctx->kernel_timing = enable != 0;
  return PAI_OK;
}

// Launch count, summed device time (ms) and summed algorithmic work of one timed kernel family since timing was enabled.
PAI_API pai_status pai_kernel_stats(pai_ctx* ctx, const char* family, int64_t* launches, double* total_ms, double* work) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_CUDA(cudaStreamSynchronize(ctx->stream));
  auto it = ctx->timed.find(family ? family : "");
  double ms = 0;
  int64_t n = 0;
  double w = 0;
  if (it != ctx->timed.end()) {
    for (size_t i = 0; i + 1 < it->second.ev.size(); i += 2) {
      float t = 0;
      PAI_CUDA(cudaEventElapsedTime(&t, it->second.ev[i], it->second.ev[i + 1]));
      ms += t;
    }
    n = it->second.launches;
    w = it->second.work;
  }
  if (launches) *launches = n;
  if (total_ms) *total_ms = ms;
  if (work) *work = w;
  return PAI_OK;
}

// ---------------------------------------------------------------- CUDA graphs
// Captures every op issued on the context between pai_graph_begin and pai_graph_end into one CUDA graph (no host
// uploads or synchronising calls in between). The device blocks the captured ops use stay reserved for the graph until
// pai_graph_destroy, so replays read and write the same memory the capture did.
PAI_API pai_status pai_graph_begin(pai_ctx* ctx) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (ctx->capture) return set_error(PAI_ERR_INVALID_OP, "a graph capture is already in progress");
  PAI_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeRelaxed));
  ctx->capture = new pai_graph();
  ctx->capture_launches0 = ctx->launches;
  return PAI_OK;
}

static void release_graph_blocks(pai_ctx* ctx, pai_graph* gr) {
  for (void* p : gr->pool.owned) ctx->graph_owner.erase(p);
  for (auto& kv : gr->pool.parked)
    for (void* p : kv.second) ctx->free_blocks[kv.first].push_back(p);
  gr->pool.owned.clear();
  gr->pool.parked.clear();
}

PAI_API pai_status pai_graph_end(pai_ctx* ctx, pai_graph** out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (!ctx->capture) return set_error(PAI_ERR_INVALID_OP, "no graph capture is in progress");
  pai_graph* gr = ctx->capture;
  ctx->capture = nullptr;
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  if (e == cudaSuccess) e = cudaGraphInstantiate(&gr->exec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    cudaGetLastError();
    release_graph_blocks(ctx, gr);
    delete gr;
    return cuda_error(e, "graph capture");
  }
  gr->launches = ctx->launches - ctx->capture_launches0;
  ctx->launches = ctx->capture_launches0;  // nothing ran yet: launches count when the graph is replayed
  *out = gr;
  return PAI_OK;
}

PAI_API pai_status pai_graph_launch(pai_ctx* ctx, pai_graph* gr) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  if (!gr || !gr->exec) return set_error(PAI_ERR_ARGUMENT, "not an instantiated graph");
  PAI_CUDA(cudaGraphLaunch(gr->exec, ctx->stream));
  ctx->launches += gr->launches;
  return PAI_OK;
}

PAI_API pai_status pai_graph_destroy(pai_ctx* ctx, pai_graph* gr) {
  if (!gr) return PAI_OK;
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_CUDA(cudaStreamSynchronize(ctx->stream));  // the last replay has finished with the reserved blocks
  if (gr->exec) cudaGraphExecDestroy(gr->exec);
  release_graph_blocks(ctx, gr);
  delete gr;
  return PAI_OK;
}

// Host -> device copy into an existing dense tensor (stream-ordered; the host buffer may be reused on return).
PAI_API pai_status pai_write(pai_ctx* ctx, const float* host, int64_t count, const pai_tensor* dst) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, dst, "destination"));
  if (!is_dense(*dst)) return set_error(PAI_ERR_ARGUMENT, "Write: the destination must be a dense tensor");
  if (count != numel(*dst))
    return set_error(PAI_ERR_ARGUMENT, "Write: %lld values for a tensor of %lld", (long long)count, (long long)numel(*dst));
  return h2d(ctx, fptr(*dst), host, (size_t)count * 4);
}
