// Fused causal GQA attention, forward and backward (online softmax; the S x L score matrix is never written to HBM).
// Replaces the composed chain of ProjectAI.Models/Modules.cs:169-203 — scores = (q·scale)·kᵀ, + causal mask
// (Modules.cs:211-218: key j visible to query i iff j <= posOffset + i), softmax over keys, ·v, heads merged to
// [B,S,H,D] — and its Autograd backward (MatMul rule Autograd.cs:54-73, Softmax rule :197-205, GQA group sum via
// ReduceGradToShape :328-341). q is scaled before the dot products exactly as Mul(q5, 1/√dh) does.
//
// This file holds the op entry points (shape checks, dispatch to the tcgen05 kernels of attention_tc.cu and
// attention_tc_bwd.cu, or to the decode kernels of attention_decode.cu) and the backward's row-dot pre-pass.
#include <math.h>

#include "common.cuh"

namespace pai {

constexpr int kMaxD = 64;

struct V4 {
  const float* p;
  int64_t s0, s1, s2, s3;
  __device__ __forceinline__ float at(int a, int b, int c, int d) const {
    return p[a * s0 + b * s1 + (int64_t)c * s2 + (int64_t)d * s3];
  }
};

struct AttnDims {
  int B, H, KVH, S, L, D, pos_offset, causal;
  float scale;
};

// ---------------------------------------------------------------- backward
// Dv[b,h,i] = Σ_d dO·O (equals Σ_j P_ij·dP_ij, the Softmax-rule dot), one warp per row.
__global__ void k_attn_dot(AttnDims a, V4 dout, const float* __restrict__ out, float* __restrict__ dv) {
  int lane = threadIdx.x & 31;
  int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t rows = (int64_t)a.B * a.H * a.S;
  if (w >= rows) return;
  int i = (int)(w % a.S);
  int h = (int)((w / a.S) % a.H);
  int b = (int)(w / ((int64_t)a.S * a.H));
  const float* orow = out + (((int64_t)b * a.S + i) * a.H + h) * a.D;
  float acc = 0.0f;
  for (int d = lane; d < a.D; d += 32) acc = fmaf(dout.at(b, i, h, d), orow[d], acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) dv[w] = acc;
}

// k_attn_dot for D % 4 == 0, D <= 64 and 16-byte aligned dout rows: a half-warp per row (lane l holds float4 l of
// the row), 32-bit row decomposition, two rows per warp.
__global__ void k_attn_dot4(AttnDims a, V4 dout, const float* __restrict__ out, float* __restrict__ dv) {
  const int half = (threadIdx.x >> 4) & 1, l = threadIdx.x & 15;
  const int64_t rows = (int64_t)a.B * a.H * a.S;
  const int64_t w = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * 2 + half;
  const bool live = w < rows;
  float acc = 0.0f;
  if (live && l < (a.D >> 2)) {
    const uint32_t r = (uint32_t)w;
    const uint32_t i = r % (uint32_t)a.S, bh = r / (uint32_t)a.S;
    const uint32_t h = bh % (uint32_t)a.H, b = bh / (uint32_t)a.H;
    const float4 g = *reinterpret_cast<const float4*>(dout.p + b * dout.s0 + i * dout.s1 + h * dout.s2 + 4 * l);
    const float4 o = *reinterpret_cast<const float4*>(out + (((int64_t)b * a.S + i) * a.H + h) * a.D + 4 * l);
    acc = fmaf(g.x, o.x, acc);
    acc = fmaf(g.y, o.y, acc);
    acc = fmaf(g.z, o.z, acc);
    acc = fmaf(g.w, o.w, acc);
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (live && l == 0) dv[w] = acc;
}

static V4 v4(const pai_tensor& t) {
  return V4{static_cast<const float*>(t.base) + t.offset, t.strides[0], t.strides[1], t.strides[2], t.strides[3]};
}

static pai_status attn_dims(const pai_tensor* q, const pai_tensor* k, const pai_tensor* v, float scale, int causal,
                            int pos_offset, AttnDims* a) {
  if (q->rank != 4 || k->rank != 4 || v->rank != 4)
    return set_error(PAI_ERR_ARGUMENT, "sdpa: q, k, v must be rank 4 ([B,H,S,D], [B,KVH,L,D])");
  a->B = q->dims[0]; a->H = q->dims[1]; a->S = q->dims[2]; a->D = q->dims[3];
  a->KVH = k->dims[1]; a->L = k->dims[2];
  a->pos_offset = pos_offset; a->causal = causal; a->scale = scale;
  for (int i = 0; i < 4; i++)
    if (k->dims[i] != v->dims[i]) return set_error(PAI_ERR_ARGUMENT, "sdpa: k and v shapes differ");
  if (k->dims[0] != a->B || k->dims[3] != a->D) return set_error(PAI_ERR_ARGUMENT, "sdpa: q and k disagree on batch or head dim");
  if (a->KVH < 1 || a->H % a->KVH) return set_error(PAI_ERR_ARGUMENT, "sdpa: heads %d not a multiple of kv heads %d", a->H, a->KVH);
  if (a->D > kMaxD) return set_error(PAI_ERR_UNSUPPORTED, "sdpa: head dim %d above %d", a->D, kMaxD);
  if (pos_offset < 0) return set_error(PAI_ERR_OUT_OF_RANGE, "sdpa: negative position offset");
  return PAI_OK;
}

// Algorithmic flops of the forward: 2 (QKᵀ) + 2 (PV) per visible (query, key) pair and head-dim element.
static double attn_fwd_flops(const AttnDims& a) {
  double pairs = 0;
  for (int i = 0; i < a.S; i++) pairs += a.causal ? (double)std::min(a.L, a.pos_offset + i + 1) : (double)a.L;
  return 4.0 * a.D * (double)a.B * a.H * pairs;
}

// attention_decode.cu
bool attn_decode_fits(const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, int H, int KVH, int S, int D);
pai_status attn_decode_fwd(pai_ctx* ctx, const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, int B, int H,
                           int KVH, int S, int L, int D, float scale, int causal, int pos_offset, float* out, float* lse,
                           const float* pos_dev = nullptr);

}  // namespace pai

using namespace pai;

pai_status attn_tc_fwd(pai_ctx* ctx, const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, int B, int H, int KVH,
                       int S, int L, int D, float scale, int causal, int pos_offset, float* out, float* lse);
pai_status attn_tc_bwd(pai_ctx* ctx, const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, const pai_tensor& dout,
                       const float* lse, const float* dvec, int B, int H, int KVH, int S, int L, int D, float scale,
                       int causal, int pos_offset, float* dq, float* dk, float* dv);

PAI_API pai_status pai_sdpa_fwd(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v, float scale,
                                int32_t causal, int32_t pos_offset, pai_tensor* out, pai_tensor* lse) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, q, "q"));
  PAI_TRY(check_view(ctx, k, "k"));
  PAI_TRY(check_view(ctx, v, "v"));
  AttnDims a;
  PAI_TRY(attn_dims(q, k, v, scale, causal, pos_offset, &a));
  int32_t od[4] = {a.B, a.S, a.H, a.D}, ld[3] = {a.B, a.H, a.S};
  pai_tensor ro, rl;
  PAI_TRY(alloc_tensor(ctx, 4, od, q->dtype, false, &ro));
  PAI_TRY(alloc_tensor(ctx, 3, ld, q->dtype, false, &rl));
  if (numel(ro) > 0 && a.L > 0 && attn_decode_fits(*q, *k, *v, a.H, a.KVH, a.S, a.D)) {
    // decode step: HBM-bound split-KV kernel (attention_decode.cu); work = K and V bytes read
    int kend = causal ? std::min(a.L, pos_offset + a.S) : a.L;
    KernelTimerScope timer(ctx, "attn_decode", 8.0 * a.B * a.KVH * (double)kend * a.D);
    PAI_TRY(attn_decode_fwd(ctx, *q, *k, *v, a.B, a.H, a.KVH, a.S, a.L, a.D, scale, causal, pos_offset, fptr(ro), fptr(rl)));
  } else if (numel(ro) > 0 && a.L > 0) {
    KernelTimerScope timer(ctx, "attn_fwd", attn_fwd_flops(a));
    PAI_TRY(attn_tc_fwd(ctx, *q, *k, *v, a.B, a.H, a.KVH, a.S, a.L, a.D, scale, causal, pos_offset, fptr(ro), fptr(rl)));
  }
  *out = ro;
  *lse = rl;
  return PAI_OK;
}

PAI_API pai_status pai_sdpa_bwd(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v,
                                const pai_tensor* out, const pai_tensor* lse, const pai_tensor* dout, float scale,
                                int32_t causal, int32_t pos_offset, pai_tensor* dq, pai_tensor* dk, pai_tensor* dv) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, q, "q"));
  PAI_TRY(check_view(ctx, k, "k"));
  PAI_TRY(check_view(ctx, v, "v"));
  PAI_TRY(check_view(ctx, out, "out"));
  PAI_TRY(check_view(ctx, lse, "lse"));
  PAI_TRY(check_view(ctx, dout, "dout"));
  AttnDims a;
  PAI_TRY(attn_dims(q, k, v, scale, causal, pos_offset, &a));
  if (dout->rank != 4 || dout->dims[0] != a.B || dout->dims[1] != a.S || dout->dims[2] != a.H || dout->dims[3] != a.D)
    return set_error(PAI_ERR_ARGUMENT, "sdpa_bwd: dout must be [B,S,H,D], got %s", shape_str(*dout).c_str());
  if (!is_dense(*out) || !is_dense(*lse)) return set_error(PAI_ERR_ARGUMENT, "sdpa_bwd: out and lse must be the forward's results");
  int32_t qd[4] = {a.B, a.H, a.S, a.D}, kd[4] = {a.B, a.KVH, a.L, a.D};
  pai_tensor rq, rk, rv;
  // the tensor-core kernels write every element of dq, dk and dv; an empty key range starts from zeros
  const bool zero = a.L == 0;
  PAI_TRY(alloc_tensor(ctx, 4, qd, q->dtype, zero, &rq));
  PAI_TRY(alloc_tensor(ctx, 4, kd, q->dtype, zero, &rk));
  PAI_TRY(alloc_tensor(ctx, 4, kd, q->dtype, zero, &rv));
  if (numel(rq) > 0 && a.L > 0) {
    Scratch dvec;
    int64_t rows = (int64_t)a.B * a.H * a.S;
    PAI_TRY(scratch(ctx, (size_t)rows * 4, &dvec));
    KernelTimerScope timer(ctx, "attn_bwd", 2.5 * attn_fwd_flops(a));
    const V4 dov = v4(*dout);
    const bool dot4 = a.D % 4 == 0 && a.D <= 64 && dov.s3 == 1 && (reinterpret_cast<uintptr_t>(dov.p) % 16 == 0) &&
                      dov.s0 % 4 == 0 && dov.s1 % 4 == 0 && dov.s2 % 4 == 0 && (reinterpret_cast<uintptr_t>(fptr(*out)) % 16 == 0) &&
                      rows < (1ll << 31);
    if (dot4)
      k_attn_dot4<<<(unsigned)((rows * 16 + 255) / 256), 256, 0, ctx->stream>>>(a, dov, fptr(*out), static_cast<float*>(dvec.p));
    else
      k_attn_dot<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, ctx->stream>>>(a, dov, fptr(*out), static_cast<float*>(dvec.p));
    PAI_LAUNCH_CHECK("sdpa_bwd dot");
    PAI_TRY(attn_tc_bwd(ctx, *q, *k, *v, *dout, fptr(*lse), static_cast<float*>(dvec.p), a.B, a.H, a.KVH, a.S, a.L, a.D,
                        scale, causal, pos_offset, fptr(rq), fptr(rk), fptr(rv)));
  }
  *dq = rq;
  *dk = rk;
  *dv = rv;
  return PAI_OK;
}
