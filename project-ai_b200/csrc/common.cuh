// Shared internals of libprojectai_cuda.so: the per-device context (streams, caching allocator, scopes),
// error reporting, and the view descriptors kernels index through.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <utility>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "projectai_cuda.h"

#define PAI_API extern "C" __attribute__((visibility("default")))

namespace pai {

// ---------------------------------------------------------------- errors
pai_status set_error(pai_status st, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
pai_status cuda_error(cudaError_t e, const char* what);

#define PAI_TRY(x) do { pai_status _s = (x); if (_s != PAI_OK) return _s; } while (0)
#define PAI_CUDA(x) do { cudaError_t _e = (x); if (_e != cudaSuccess) return ::pai::cuda_error(_e, #x); } while (0)
// A launch through launch_pdl: reports its error and counts the launch on the context.
#define PAI_PDL_LAUNCH(call, what)                                      \
  do {                                                                  \
    cudaError_t _e = (call);                                            \
    if (_e != cudaSuccess) return ::pai::cuda_error(_e, what);          \
    ctx->launches++;                                                    \
  } while (0)
// Every kernel launch site ends with this: it reports launch errors and counts the launch on the context.
#define PAI_LAUNCH_CHECK(what)                                          \
  do {                                                                  \
    cudaError_t _e = cudaGetLastError();                                \
    if (_e != cudaSuccess) return ::pai::cuda_error(_e, what);          \
    ctx->launches++;                                                    \
  } while (0)

// ---------------------------------------------------------------- context
struct BlockInfo {
  size_t bytes;      // rounded size held from the cache
  int scope;         // index of the owning open scope, or -1
};

struct NcclState;  // defined in dp.cu
struct IoState;    // defined in io.cu

// Device blocks a captured CUDA graph reads or writes. They stay reserved while the graph exists: blocks freed during
// or after the capture are parked here instead of returning to the allocator's cache.
struct GraphPool {
  std::unordered_set<void*> owned;
  std::unordered_map<size_t, std::vector<void*>> parked;  // rounded size -> owned blocks not currently live
};

}  // namespace pai

struct pai_graph {
  cudaGraphExec_t exec = nullptr;
  pai::GraphPool pool;
  int64_t launches = 0;  // kernel launches captured (counted again on every replay)
};

struct pai_ctx {
  int device = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;       // compute stream: every op is ordered here
  cudaStream_t comm_stream = nullptr;  // data-parallel all-reduce stream
  std::recursive_mutex mu;
  // caching allocator: rounded size -> free device blocks
  std::unordered_map<size_t, std::vector<void*>> free_blocks;
  std::unordered_map<void*, pai::BlockInfo> live;
  std::vector<std::unordered_set<void*>> scopes;
  int64_t in_use = 0, peak = 0, reserved = 0;
  // device flag the kernels with bounded waits report into (0 = ok)
  int* d_error_flag = nullptr;
  pai::NcclState* nccl = nullptr;
  pai::IoState* io = nullptr;  // checkpoint streaming and the open packed dataset (io.cu)
  char name[128] = {0};
  // instrumentation: kernel launches issued, a stream timer, and per-kernel-family event timing
  int64_t launches = 0;
  cudaEvent_t timer_start = nullptr, timer_stop = nullptr;
  bool kernel_timing = false;
  struct Timed {
    std::vector<cudaEvent_t> ev;  // start/stop pairs
    double work = 0;              // algorithmic flops or bytes of the timed launches
    int64_t launches = 0;
  };
  std::unordered_map<std::string, Timed> timed;
  std::vector<cudaEvent_t> event_pool;
  // pinned staging ring for small host->device uploads (ids, targets, batch offsets): copies from pinned memory are
  // truly asynchronous, so an op's small uploads never stall the stream
  char* pinned = nullptr;
  cudaEvent_t pinned_ev[32] = {};
  int pinned_next = 0;
  // CUDA graph capture: the graph being captured, and which live graph owns each reserved block
  pai_graph* capture = nullptr;
  int64_t capture_launches0 = 0;
  std::unordered_map<void*, pai_graph*> graph_owner;
  // kernels whose dynamic shared-memory limit was raised on this context's device, with the bytes set
  std::unordered_map<const void*, int> smem_attr;
  // two-CTA clusters of the CTA-pair GEMM resident at once on this device (0: not queried yet, -1: unavailable)
  int gemm_pair_slots = 0;
};

namespace pai {
// Raises a kernel's dynamic shared-memory limit to `bytes`. The attribute belongs to the device that is current (a
// CUDA context per device), so it is set once per library context, which is bound to one device and entered (device
// made current) by every entry point, and only under the context's lock.
template <class Kernel>
inline cudaError_t smem_limit(pai_ctx* ctx, Kernel* kernel, int bytes) {
  const void* key = reinterpret_cast<const void*>(kernel);
  auto it = ctx->smem_attr.find(key);
  if (it != ctx->smem_attr.end() && it->second >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) ctx->smem_attr[key] = bytes;
  return e;
}

// Brackets one launch with events on the compute stream when kernel timing is on (pai_kernel_timing).
struct KernelTimerScope {
  pai_ctx* ctx;
  pai_ctx::Timed* slot = nullptr;
  KernelTimerScope(pai_ctx* c, const char* family, double work);
  ~KernelTimerScope();
};
}  // namespace pai

namespace pai {

// Makes ctx's device current on the calling thread (the contract may be driven from any thread).
pai_status enter(pai_ctx* ctx);

// Stream-ordered caching allocator. Blocks return to the cache on free and are reused by later work on the same
// compute stream, so reuse never races with a kernel still reading the block.
pai_status raw_alloc(pai_ctx* ctx, size_t bytes, void** out);
void raw_free(pai_ctx* ctx, void* p);

// Allocates a contiguous tensor registered in the innermost scope. zero != 0 clears it on the stream.
pai_status alloc_tensor(pai_ctx* ctx, int rank, const int32_t* dims, int dtype, bool zero, pai_tensor* out);
// A scratch buffer that is not a tensor: freed by the caller with raw_free (stream-ordered).
struct Scratch {
  pai_ctx* ctx = nullptr;
  void* p = nullptr;
  ~Scratch() { if (p) raw_free(ctx, p); }
};
pai_status scratch(pai_ctx* ctx, size_t bytes, Scratch* s);

// Host -> device copy of a small host array into a stream-ordered scratch block.
pai_status upload(pai_ctx* ctx, const void* host, size_t bytes, Scratch* s);
// Stream-ordered host -> device copy; buffers up to kPinnedChunk bytes go through the pinned staging ring.
constexpr size_t kPinnedChunk = 256 * 1024;
constexpr int kPinnedChunks = 32;
pai_status h2d(pai_ctx* ctx, void* dst, const void* host, size_t bytes);

// ---------------------------------------------------------------- views
int64_t numel(const pai_tensor& t);
std::string shape_str(const pai_tensor& t);
bool is_dense(const pai_tensor& t);  // contiguous row-major (offset may be non-zero)
pai_status check_view(pai_ctx* ctx, const pai_tensor* t, const char* what);
void set_contiguous(pai_tensor* t, void* base, int rank, const int32_t* dims, int dtype);
pai_tensor broadcast_view(const pai_tensor& t, int rank, const int32_t* dims);
bool broadcast_shape(const pai_tensor& a, const pai_tensor& b, int* rank, int32_t* dims);
inline int norm_axis(int axis, int rank) { return axis < 0 ? axis + rank : axis; }

// A view reduced for indexing on the device: size-1 axes dropped, mergeable neighbours merged.
struct DView {
  int64_t offset;
  int32_t rank;
  int32_t dims[PAI_MAX_RANK];
  int64_t strides[PAI_MAX_RANK];
};
// Collapses n views that share one logical shape (dims) jointly, so one flat index addresses all of them.
void collapse(int rank, const int32_t* dims, const pai_tensor* const* views, int n, DView* out);

inline float* fptr(const pai_tensor& t) { return static_cast<float*>(t.base) + t.offset; }

// Programmatic dependent launch for the decode-step kernels: a kernel launched with launch_pdl may start while the
// previous kernel on the stream is still running. It must call pdl_wait() before it reads anything an earlier
// kernel wrote (and before it exits); work that only reads data written before (weights, caches of earlier steps)
// may be issued first. pdl_trigger() lets the next such kernel launch early.

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl with thread-block clusters of cluster_x CTAs along x (grid.x must be a multiple of cluster_x).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                               unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Grid size for a grid-stride loop: at most `waves` resident waves of `threads`-thread blocks.
inline int grid_for(pai_ctx* ctx, int64_t n, int threads, int per_thread = 1, int waves = 8) {
  int64_t want = (n + (int64_t)threads * per_thread - 1) / ((int64_t)threads * per_thread);
  int64_t cap = (int64_t)ctx->sm_count * waves;
  if (want < 1) want = 1;
  return (int)(want < cap ? want : cap);
}

}  // namespace pai

// Logical row-major index -> element offset of a collapsed view.
// The loops below run over the fixed maximum rank with constant indices (the inactive dims are skipped): a loop
// bounded by v.rank indexes the kernel parameter arrays dynamically, which copies them to per-thread local memory.
__device__ __forceinline__ int64_t dview_offset(const pai::DView& v, int64_t i) {
  int64_t off = v.offset;
#pragma unroll
  for (int d = PAI_MAX_RANK - 1; d >= 0; d--) {
    if (d < v.rank) {
      int64_t dim = v.dims[d];
      int64_t q = i / dim;
      off += (i - q * dim) * v.strides[d];
      i = q;
    }
  }
  return off;
}

__device__ __forceinline__ int64_t dview_offset32(const pai::DView& v, uint32_t i) {
  int64_t off = v.offset;
#pragma unroll
  for (int d = PAI_MAX_RANK - 1; d >= 0; d--) {
    if (d < v.rank) {
      uint32_t dim = (uint32_t)v.dims[d];
      uint32_t q = i / dim;
      off += (int64_t)(i - q * dim) * v.strides[d];
      i = q;
    }
  }
  return off;
}

// Row r of up to three jointly collapsed views (same dims): one 32-bit coordinate decomposition, three offsets.
__device__ __forceinline__ void row_offsets3(const pai::DView& a, const pai::DView& b, const pai::DView& c, uint32_t r,
                                             int64_t& oa, int64_t& ob, int64_t& oc) {
  oa = a.offset;
  ob = b.offset;
  oc = c.offset;
#pragma unroll
  for (int d = PAI_MAX_RANK - 1; d >= 0; d--) {
    if (d < a.rank) {
      uint32_t dim = (uint32_t)a.dims[d];
      uint32_t q = r / dim;
      int64_t i = (int64_t)(r - q * dim);
      oa += i * a.strides[d];
      ob += i * b.strides[d];
      oc += i * c.strides[d];
      r = q;
    }
  }
}

// Device side of launch_pdl: wait for the previous kernel's completion (and its memory), and allow the next kernel
// to launch. Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// SiLU(g)·u with the element operations of the reference's Sigmoid (sign-split, CpuComputeBackend.cs:304-317), SiLU
// (x·sigmoid(x), :385-391) and Mul, each rounded once: shared by the SwiGLU kernel and the fused decode epilogue.
// The two branches share one exponential, expf(-|g|) (= expf(-g) for g >= 0 and expf(g) otherwise, exactly), so a
// warp whose elements differ in sign evaluates it once per element; the quotients are the branches' own.
__device__ __forceinline__ float silu_mul_value(float g, float u) {
  const float t = expf(-fabsf(g));
  const float s = __fdiv_rn(g >= 0.0f ? 1.0f : t, __fadd_rn(1.0f, t));
  return __fmul_rn(__fmul_rn(g, s), u);
}

// Internal launchers shared across translation units.
namespace pai {
// dst (dense, element offset dst_off in buffer dst_base) <- logical elements of src view.
pai_status gather_dense(pai_ctx* ctx, const pai_tensor& src, float* dst);
// Makes `t` dense: returns t itself if already dense, else a gathered copy held in `holder`.
pai_status dense_input(pai_ctx* ctx, const pai_tensor& t, const float** out, Scratch* holder);
}  // namespace pai
