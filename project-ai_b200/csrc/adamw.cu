// Fused AdamW: one pass over p, g, m, v (28 bytes per element) in place of the ~15 allocating backend ops of
// ProjectAI.Core/Optimizers.cs:81-123. Every element follows the reference's operation order, and the host-side
// scalars (1-β, 1/(1-β^t), lr·wd) are formed exactly as the reference forms them in float, so the update is
// bit-identical to the composed reference ops.
#include <math.h>

#include "common.cuh"

namespace pai {

struct AdamScalars {
  float b1, b2, one_m_b1, one_m_b2, inv_bc1, inv_bc2, eps, lr, lr_wd, grad_scale;
  int scale_grad;
};

__device__ __forceinline__ void adam_elem(float& p, float gr, float& m, float& v, const AdamScalars& s) {
  float g = s.scale_grad ? __fmul_rn(gr, s.grad_scale) : gr;
  // m = β1·m + (1−β1)·g ;  v = β2·v + (1−β2)·g²
  float mn = __fadd_rn(__fmul_rn(m, s.b1), __fmul_rn(g, s.one_m_b1));
  float vn = __fadd_rn(__fmul_rn(v, s.b2), __fmul_rn(__fmul_rn(g, g), s.one_m_b2));
  float mhat = __fmul_rn(mn, s.inv_bc1);
  float vhat = __fmul_rn(vn, s.inv_bc2);
  float adaptive = __fdiv_rn(mhat, __fadd_rn(__fsqrt_rn(vhat), s.eps));
  // θ ← θ − (lr·adaptive + (lr·λ)·θ)
  float delta = __fadd_rn(__fmul_rn(adaptive, s.lr), __fmul_rn(p, s.lr_wd));
  p = __fsub_rn(p, delta);
  m = mn;
  v = vn;
}

__global__ void k_adamw(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                        int64_t n, AdamScalars s, bool vec) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    int64_t n4 = n >> 2;
    float4* p4 = reinterpret_cast<float4*>(p);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    for (int64_t i = tid; i < n4; i += stride) {
      float4 pp = p4[i], gg = g4[i], mm = m4[i], vv = v4[i];
      adam_elem(pp.x, gg.x, mm.x, vv.x, s);
      adam_elem(pp.y, gg.y, mm.y, vv.y, s);
      adam_elem(pp.z, gg.z, mm.z, vv.z, s);
      adam_elem(pp.w, gg.w, mm.w, vv.w, s);
      p4[i] = pp; m4[i] = mm; v4[i] = vv;
    }
    for (int64_t i = (n4 << 2) + tid; i < n; i += stride) adam_elem(p[i], g[i], m[i], v[i], s);
  } else {
    for (int64_t i = tid; i < n; i += stride) adam_elem(p[i], g[i], m[i], v[i], s);
  }
}

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_adamw_step(pai_ctx* ctx, const pai_tensor* p, const pai_tensor* g, const pai_tensor* m,
                                  const pai_tensor* v, float lr, float beta1, float beta2, float eps, float wd, int32_t t,
                                  float grad_scale) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, p, "param"));
  PAI_TRY(check_view(ctx, g, "grad"));
  PAI_TRY(check_view(ctx, m, "m"));
  PAI_TRY(check_view(ctx, v, "v"));
  int64_t n = numel(*p);
  if (numel(*g) != n || numel(*m) != n || numel(*v) != n)
    return set_error(PAI_ERR_ARGUMENT, "AdamWStep: param, grad and moments must have equal element counts");
  if (!is_dense(*p) || !is_dense(*g) || !is_dense(*m) || !is_dense(*v))
    return set_error(PAI_ERR_ARGUMENT, "AdamWStep: tensors must be contiguous");
  if (t < 1) return set_error(PAI_ERR_OUT_OF_RANGE, "AdamWStep: timestep must be >= 1");
  if (n == 0) return PAI_OK;
  AdamScalars s;
  s.b1 = beta1;
  s.b2 = beta2;
  s.one_m_b1 = 1.0f - beta1;
  s.one_m_b2 = 1.0f - beta2;
  float bc1 = 1.0f - powf(beta1, (float)t);  // MathF.Pow(Beta1, t)
  float bc2 = 1.0f - powf(beta2, (float)t);
  s.inv_bc1 = 1.0f / bc1;
  s.inv_bc2 = 1.0f / bc2;
  s.eps = eps;
  s.lr = lr;
  s.lr_wd = lr * wd;
  s.grad_scale = grad_scale;
  s.scale_grad = grad_scale != 1.0f;
  float *pp = fptr(*p), *mp = fptr(*m), *vp = fptr(*v);
  const float* gp = fptr(*g);
  bool vec = ((reinterpret_cast<uintptr_t>(pp) | reinterpret_cast<uintptr_t>(gp) | reinterpret_cast<uintptr_t>(mp) |
               reinterpret_cast<uintptr_t>(vp)) & 15) == 0;
  k_adamw<<<grid_for(ctx, n, 256, vec ? 4 : 1, 4), 256, 0, ctx->stream>>>(pp, gp, mp, vp, n, s, vec);
  PAI_LAUNCH_CHECK("adamw");
  return PAI_OK;
}
