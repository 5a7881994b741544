// Elementwise ops with NumPy broadcasting and strided inputs.
// Contract: IComputeBackend.cs:20-31; semantics CpuComputeBackend.cs:86-156 (binary ops and scalar ops are IEEE
// single operations, so these kernels are bit-exact with the oracle), :304-317 (sign-split sigmoid), :385-391 (SiLU).
#include "common.cuh"

namespace pai {

enum BinKind { kAdd = 0, kSub = 1, kMul = 2, kDiv = 3 };

template <int K>
__device__ __forceinline__ float binop(float x, float y) {
  if (K == kAdd) return __fadd_rn(x, y);
  if (K == kSub) return __fsub_rn(x, y);
  if (K == kMul) return __fmul_rn(x, y);
  return __fdiv_rn(x, y);
}

// Dense, same-shape operands: 128-bit loads when every pointer is 16-byte aligned.
template <int K>
__global__ void k_binary_dense(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o, int64_t n,
                               bool vec) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    int64_t n4 = n >> 2;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    float4* o4 = reinterpret_cast<float4*>(o);
    for (int64_t i = tid; i < n4; i += stride) {
      float4 x = a4[i], y = b4[i], z;
      z.x = binop<K>(x.x, y.x); z.y = binop<K>(x.y, y.y); z.z = binop<K>(x.z, y.z); z.w = binop<K>(x.w, y.w);
      o4[i] = z;
    }
    for (int64_t i = (n4 << 2) + tid; i < n; i += stride) o[i] = binop<K>(a[i], b[i]);
  } else {
    for (int64_t i = tid; i < n; i += stride) o[i] = binop<K>(a[i], b[i]);
  }
}

// b broadcast along the leading axes of a dense a: o[r, c] = a[r, c] op b[c] (bias-style, the common GQA/norm case).
template <int K>
__global__ void k_binary_rowbcast(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o,
                                  int64_t n, int64_t inner, bool b_first) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float x = a[i], y = b[i % inner];
    o[i] = b_first ? binop<K>(y, x) : binop<K>(x, y);
  }
}

template <int K>
__global__ void k_binary_strided(const float* __restrict__ a, DView av, const float* __restrict__ b, DView bv,
                                 float* __restrict__ o, int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (n < (1ll << 31)) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
      o[i] = binop<K>(a[dview_offset32(av, (uint32_t)i)], b[dview_offset32(bv, (uint32_t)i)]);
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
      o[i] = binop<K>(a[dview_offset(av, i)], b[dview_offset(bv, i)]);
  }
}

template <int K>
static pai_status launch_binary(pai_ctx* ctx, const pai_tensor& a, const pai_tensor& b, const pai_tensor& out) {
  int64_t n = numel(out);
  if (n == 0) return PAI_OK;
  float* o = fptr(out);
  pai_tensor av = broadcast_view(a, out.rank, out.dims), bv = broadcast_view(b, out.rank, out.dims);
  const pai_tensor* views[3] = {&av, &bv, &out};
  DView dv[3];
  collapse(out.rank, out.dims, views, 3, dv);
  const float* pa = static_cast<const float*>(a.base);
  const float* pb = static_cast<const float*>(b.base);
  int threads = 256;
  auto is_flat = [](const DView& v) { return v.rank == 0 || (v.rank == 1 && v.strides[0] == 1); };
  if (is_flat(dv[0]) && is_flat(dv[1])) {
    const float* x = pa + dv[0].offset;
    const float* y = pb + dv[1].offset;
    bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(o)) & 15) == 0;
    k_binary_dense<K><<<grid_for(ctx, n, threads, vec ? 4 : 1), threads, 0, ctx->stream>>>(x, y, o, n, vec);
  } else if (dv[0].rank == 2 && dv[0].strides[0] == dv[0].dims[1] && dv[0].strides[1] == 1 && dv[1].strides[0] == 0 &&
             dv[1].strides[1] == 1) {
    k_binary_rowbcast<K><<<grid_for(ctx, n, threads), threads, 0, ctx->stream>>>(pa + dv[0].offset, pb + dv[1].offset, o, n,
                                                                                dv[0].dims[1], false);
  } else if (dv[1].rank == 2 && dv[1].strides[0] == dv[1].dims[1] && dv[1].strides[1] == 1 && dv[0].strides[0] == 0 &&
             dv[0].strides[1] == 1) {
    k_binary_rowbcast<K><<<grid_for(ctx, n, threads), threads, 0, ctx->stream>>>(pb + dv[1].offset, pa + dv[0].offset, o, n,
                                                                                dv[1].dims[1], true);
  } else {
    k_binary_strided<K><<<grid_for(ctx, n, threads), threads, 0, ctx->stream>>>(pa, dv[0], pb, dv[1], o, n);
  }
  PAI_LAUNCH_CHECK("binary op");
  return PAI_OK;
}

static pai_status binary(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, pai_tensor* out, int kind) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, a, "a"));
  PAI_TRY(check_view(ctx, b, "b"));
  int rank;
  int32_t dims[PAI_MAX_RANK];
  if (!broadcast_shape(*a, *b, &rank, dims))
    return set_error(PAI_ERR_ARGUMENT, "Shapes %s and %s are not broadcast-compatible.", shape_str(*a).c_str(),
                     shape_str(*b).c_str());
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, rank, dims, a->dtype, false, &r));
  pai_status st;
  switch (kind) {
    case kAdd: st = launch_binary<kAdd>(ctx, *a, *b, r); break;
    case kSub: st = launch_binary<kSub>(ctx, *a, *b, r); break;
    case kMul: st = launch_binary<kMul>(ctx, *a, *b, r); break;
    default: st = launch_binary<kDiv>(ctx, *a, *b, r); break;
  }
  if (st != PAI_OK) return st;
  *out = r;
  return PAI_OK;
}

// ---------------------------------------------------------------- unary
enum UnKind { kAddS = 0, kMulS = 1, kSqrt = 2, kSigmoid = 3, kSilu = 4 };

// CpuComputeBackend.SigmoidScalar (CpuComputeBackend.cs:312-317).
__device__ __forceinline__ float sigmoid_f(float v) {
  if (v >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
  float t = expf(v);
  return __fdiv_rn(t, __fadd_rn(1.0f, t));
}

template <int K>
__device__ __forceinline__ float unop(float v, float s) {
  if (K == kAddS) return __fadd_rn(v, s);
  if (K == kMulS) return __fmul_rn(v, s);
  if (K == kSqrt) return __fsqrt_rn(v);
  if (K == kSigmoid) return sigmoid_f(v);
  return __fmul_rn(v, sigmoid_f(v));
}

template <int K>
__global__ void k_unary_dense(const float* __restrict__ x, float* __restrict__ o, int64_t n, float s, bool vec) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    int64_t n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* o4 = reinterpret_cast<float4*>(o);
    for (int64_t i = tid; i < n4; i += stride) {
      float4 v = x4[i];
      v.x = unop<K>(v.x, s); v.y = unop<K>(v.y, s); v.z = unop<K>(v.z, s); v.w = unop<K>(v.w, s);
      o4[i] = v;
    }
    for (int64_t i = (n4 << 2) + tid; i < n; i += stride) o[i] = unop<K>(x[i], s);
  } else {
    for (int64_t i = tid; i < n; i += stride) o[i] = unop<K>(x[i], s);
  }
}

template <int K>
__global__ void k_unary_strided(const float* __restrict__ x, DView xv, float* __restrict__ o, int64_t n, float s) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    o[i] = unop<K>(x[dview_offset(xv, i)], s);
}

template <int K>
static pai_status unary(pai_ctx* ctx, const pai_tensor* x, float s, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, x->rank, x->dims, x->dtype, false, &r));
  int64_t n = numel(r);
  if (n > 0) {
    float* o = fptr(r);
    if (is_dense(*x)) {
      const float* xp = fptr(*x);
      bool vec = ((reinterpret_cast<uintptr_t>(xp) | reinterpret_cast<uintptr_t>(o)) & 15) == 0;
      k_unary_dense<K><<<grid_for(ctx, n, 256, vec ? 4 : 1), 256, 0, ctx->stream>>>(xp, o, n, s, vec);
    } else {
      const pai_tensor* v[1] = {x};
      DView xv;
      collapse(x->rank, x->dims, v, 1, &xv);
      xv.offset = 0;
      k_unary_strided<K><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(fptr(*x), xv, o, n, s);
    }
    PAI_LAUNCH_CHECK("unary op");
  }
  *out = r;
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_add(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return binary(c, a, b, o, kAdd); }
PAI_API pai_status pai_sub(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return binary(c, a, b, o, kSub); }
PAI_API pai_status pai_mul(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return binary(c, a, b, o, kMul); }
PAI_API pai_status pai_div(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return binary(c, a, b, o, kDiv); }
PAI_API pai_status pai_add_scalar(pai_ctx* c, const pai_tensor* a, float s, pai_tensor* o) { return unary<kAddS>(c, a, s, o); }
PAI_API pai_status pai_mul_scalar(pai_ctx* c, const pai_tensor* a, float s, pai_tensor* o) { return unary<kMulS>(c, a, s, o); }
PAI_API pai_status pai_sqrt(pai_ctx* c, const pai_tensor* x, pai_tensor* o) { return unary<kSqrt>(c, x, 0.f, o); }
PAI_API pai_status pai_sigmoid(pai_ctx* c, const pai_tensor* x, pai_tensor* o) { return unary<kSigmoid>(c, x, 0.f, o); }
PAI_API pai_status pai_silu(pai_ctx* c, const pai_tensor* x, pai_tensor* o) { return unary<kSilu>(c, x, 0.f, o); }
