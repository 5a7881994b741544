// pai_rmsnorm_bwd_noalloc: the RMSNorm backward for callers that cannot allocate device memory.
//
// Some callers must not call cudaMalloc: a serving or training process that reserves all GPU memory for its own
// pools at start-up, code that must not trigger the device-wide synchronisation an allocation can cause, or a host
// that hands this library only buffers it owns. The regular pai_rmsnorm_bwd allocates its outputs and a scratch
// buffer of per-block dw partials through the context's caching allocator. This variant writes into output
// tensors the caller supplies and keeps its scratch in a fixed file-scope device array (kNoAllocScratchFloats
// floats, 4 MiB), which every GPU that loads the library holds until the process exits.
//
// Properties the caller relies on:
//  * It calls no cudaMalloc, cudaFree or other allocating routine, and it does not use the context's allocator.
//  * The first call on a device resolves the array's device address with cudaGetSymbolAddress (with that device
//    current) and caches it. Make that first call before any stream capture on the device.
//  * All calls share the one array, so calls whose kernels overlap on the GPU (different streams, or different
//    contexts of one device) race on it. Calls ordered on one stream are safe: each call overwrites every scratch
//    element it later reads, so nothing has to start at zero.
//  * Limits: the row length d must be at most kNoAllocMaxD (8192); inputs and outputs must be dense F32 tensors.
#include <mutex>

#include "common.cuh"

namespace pai {

constexpr int kNoAllocMaxD = 8192;
constexpr int kNoAllocMaxBlocks = 128;
constexpr size_t kNoAllocScratchFloats = (size_t)kNoAllocMaxD * kNoAllocMaxBlocks;  // 4 MiB

// Per-block dw partials of the RMSNorm backward ([blocks, d], blocks <= kNoAllocMaxBlocks).
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// The kernels of the regular RMSNorm backward (nn.cu).
__global__ void k_rmsnorm_bwd(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ g,
                              float* __restrict__ dx, float* __restrict__ dw_part, int64_t rows, int d, float eps,
                              int rows_per_block);
__global__ void k_colsum(const float* __restrict__ part, float* __restrict__ out, int parts, int d);

// Device address of g_noalloc_scratch per device ordinal, resolved once with that device current.
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {};

static pai_status noalloc_scratch(int device, float** out) {
  if (device < 0 || device >= 64) return set_error(PAI_ERR_OUT_OF_RANGE, "device ordinal %d not supported", device);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_ptr[device] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[device];
  return PAI_OK;
}

static pai_status need_dense(pai_ctx* ctx, const pai_tensor* t, const char* what) {
  PAI_TRY(check_view(ctx, t, what));
  if (!is_dense(*t)) return set_error(PAI_ERR_ARGUMENT, "%s: the allocation-free RMSNorm backward needs dense tensors", what);
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_rmsnorm_bwd_noalloc(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* w, const pai_tensor* g,
                                           float eps, const pai_tensor* dx, const pai_tensor* dw) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(need_dense(ctx, x, "x"));
  PAI_TRY(need_dense(ctx, w, "weight"));
  PAI_TRY(need_dense(ctx, g, "grad"));
  PAI_TRY(need_dense(ctx, dx, "dx"));
  PAI_TRY(need_dense(ctx, dw, "dw"));
  if (x->rank == 0) return set_error(PAI_ERR_ARGUMENT, "RmsNorm requires rank >= 1.");
  int d = x->dims[x->rank - 1];
  int64_t n = numel(*x);
  if (w->rank != 1 || w->dims[0] != d || numel(*g) != n || numel(*dx) != n || numel(*dw) != d)
    return set_error(PAI_ERR_ARGUMENT, "RmsNormBackward: shapes disagree (x %s, weight %s, grad %s, dx %s, dw %s)",
                     shape_str(*x).c_str(), shape_str(*w).c_str(), shape_str(*g).c_str(), shape_str(*dx).c_str(),
                     shape_str(*dw).c_str());
  if (d > kNoAllocMaxD)
    return set_error(PAI_ERR_OUT_OF_RANGE, "RmsNormBackward without allocation supports rows of at most %d elements; got %d",
                     kNoAllocMaxD, d);
  if (d == 0 || n == 0) return PAI_OK;
  float* part = nullptr;
  PAI_TRY(noalloc_scratch(ctx->device, &part));
  int64_t rows = n / d;
  int threads = 256, nw = threads / 32;
  size_t smem = (size_t)nw * d * 4;
  if (smem > 200 * 1024) { threads = 64; nw = 2; smem = (size_t)nw * d * 4; }
  int blocks = kNoAllocMaxBlocks < ctx->sm_count ? kNoAllocMaxBlocks : ctx->sm_count;
  int rpb = (int)((rows + blocks - 1) / blocks);
  if (rpb < nw) rpb = nw;
  blocks = (int)((rows + rpb - 1) / rpb);  // <= kNoAllocMaxBlocks, so blocks * d fits the array
  if (smem > 48 * 1024) PAI_CUDA(smem_limit(ctx, k_rmsnorm_bwd, (int)smem));
  k_rmsnorm_bwd<<<blocks, threads, smem, ctx->stream>>>(fptr(*x), fptr(*w), fptr(*g), fptr(*dx), part, rows, d, eps, rpb);
  PAI_LAUNCH_CHECK("rmsnorm_bwd (no allocation)");
  k_colsum<<<(d + 255) / 256, 256, 0, ctx->stream>>>(part, fptr(*dw), blocks, d);
  PAI_LAUNCH_CHECK("rmsnorm_bwd colsum (no allocation)");
  return PAI_OK;
}
