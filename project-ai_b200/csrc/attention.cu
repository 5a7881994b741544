// Fused causal GQA attention, forward and backward (online softmax; the S x L score matrix is never written to HBM).
// Replaces the composed chain of ProjectAI.Models/Modules.cs:169-203 — scores = (q·scale)·kᵀ, + causal mask
// (Modules.cs:211-218: key j visible to query i iff j <= posOffset + i), softmax over keys, ·v, heads merged to
// [B,S,H,D] — and its Autograd backward (MatMul rule Autograd.cs:54-73, Softmax rule :197-205, GQA group sum via
// ReduceGradToShape :328-341). q is scaled before the dot products exactly as Mul(q5, 1/√dh) does.
//
// Tiling: 64 queries x 64 keys per step, 256 threads as a 16x16 grid, each thread a 4x4 sub-tile; head dim <= 64
// (zero-padded in shared memory). fp32 FMA on the CUDA cores.
#include <math.h>

#include "common.cuh"

namespace pai {

constexpr int kT = 64;        // tile rows / cols
constexpr int kP = kT + 4;    // padded pitch (floats), keeps float4 alignment
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

__device__ __forceinline__ float rowmax16(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float rowsum16(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Loads rows [r0, r0+64) x D of a 4-D view at (b, h, row, d) into smem, d-major (t[d][r]) and/or row-major (t[r][d]).
__device__ __forceinline__ void load_tile(const V4& v, int b, int h, int r0, int rows, int D, float mul, float* dmaj,
                                          float* rmaj) {
  for (int idx = threadIdx.x; idx < kT * kMaxD; idx += blockDim.x) {
    int r = idx / kMaxD, d = idx % kMaxD;
    float x = (r0 + r < rows && d < D) ? v.at(b, h, r0 + r, d) : 0.0f;
    if (mul != 1.0f) x = __fmul_rn(x, mul);
    if (dmaj) dmaj[d * kP + r] = x;
    if (rmaj) rmaj[r * kP + d] = x;
  }
}

// S[i][j] = Σ_d A[d][4ty+i]·B[d][4tx+j] over d-major tiles.
__device__ __forceinline__ void tile_dot(const float* A, const float* Bm, int D, int ty, int tx, float s[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) s[i][j] = 0.0f;
  for (int d = 0; d < D; d++) {
    float4 a = *reinterpret_cast<const float4*>(A + d * kP + 4 * ty);
    float4 b = *reinterpret_cast<const float4*>(Bm + d * kP + 4 * tx);
    float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) s[i][j] = fmaf(av[i], bv[j], s[i][j]);
  }
}

// acc[i][j] += Σ_r X[r][4ty+i]·Y[r][4tx+j] over row-major tiles (r = 0..63).
__device__ __forceinline__ void tile_acc(const float* X, const float* Y, float acc[4][4]) {
#pragma unroll 8
  for (int r = 0; r < kT; r++) {
    float4 a = *reinterpret_cast<const float4*>(X + r * kP + 4 * (threadIdx.x >> 4));
    float4 b = *reinterpret_cast<const float4*>(Y + r * kP + 4 * (threadIdx.x & 15));
    float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
  }
}

__device__ __forceinline__ bool visible(const AttnDims& a, int qi, int kj) {
  return kj < a.L && (!a.causal || kj <= a.pos_offset + qi);
}

// ---------------------------------------------------------------- forward
__global__ void __launch_bounds__(256) k_attn_fwd(AttnDims a, V4 q, V4 k, V4 v, float* __restrict__ out,
                                                  float* __restrict__ lse) {
  extern __shared__ float sm[];
  float* Qt = sm;               // [d][r]
  float* Kt = Qt + kMaxD * kP;  // [d][c]
  float* Vs = Kt + kMaxD * kP;  // [c][d]
  float* Ps = Vs + kT * kP;     // [c][r]
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * kT;
  const int kvh = h / (a.H / a.KVH);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  load_tile(q, b, h, q0, a.S, a.D, a.scale, Qt, nullptr);
  float m[4], l[4], o[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    m[i] = -INFINITY; l[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; j++) o[i][j] = 0.0f;
  }
  int kend = a.L;
  if (a.causal) kend = min(a.L, a.pos_offset + q0 + kT);
  for (int k0 = 0; k0 < kend; k0 += kT) {
    __syncthreads();
    load_tile(k, b, kvh, k0, a.L, a.D, 1.0f, Kt, nullptr);
    load_tile(v, b, kvh, k0, a.L, a.D, 1.0f, nullptr, Vs);
    __syncthreads();
    float s[4][4];
    tile_dot(Qt, Kt, a.D, ty, tx, s);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      int qi = q0 + 4 * ty + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        if (!visible(a, qi, k0 + 4 * tx + j)) s[i][j] = -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
      mx = rowmax16(mx);
      float mn = fmaxf(m[i], mx);
      float alpha = (m[i] == -INFINITY) ? 0.0f : expf(m[i] - mn);
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        float p = (s[i][j] == -INFINITY) ? 0.0f : expf(s[i][j] - mn);
        s[i][j] = p;
        rs += p;
      }
      rs = rowsum16(rs);
      l[i] = l[i] * alpha + rs;
      m[i] = mn;
#pragma unroll
      for (int j = 0; j < 4; j++) o[i][j] *= alpha;
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) Ps[(4 * tx + j) * kP + 4 * ty + i] = s[i][j];
    __syncthreads();
    tile_acc(Ps, Vs, o);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int qi = q0 + 4 * ty + i;
    if (qi >= a.S) continue;
    float inv = 1.0f / l[i];
    float* orow = out + (((int64_t)b * a.S + qi) * a.H + h) * a.D;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int d = 4 * tx + j;
      if (d < a.D) orow[d] = o[i][j] * inv;
    }
    if (tx == 0) lse[((int64_t)b * a.H + h) * a.S + qi] = m[i] + logf(l[i]);
  }
}

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

// dK, dV for one 64-key tile of one KV head, summed over the GQA group and all query tiles that see it.
__global__ void __launch_bounds__(256) k_attn_bwd_kv(AttnDims a, V4 q, V4 k, V4 v, V4 dout, const float* __restrict__ lse,
                                                     const float* __restrict__ dvec, float* __restrict__ dk,
                                                     float* __restrict__ dvv) {
  extern __shared__ float sm[];
  float* Kt = sm;                 // [d][c]
  float* Vt = Kt + kMaxD * kP;    // [d][c]
  float* Qt = Vt + kMaxD * kP;    // [d][r]  (scaled q)
  float* dOt = Qt + kMaxD * kP;   // [d][r]
  float* Qr = dOt + kMaxD * kP;   // [r][d]  (scaled q)
  float* dOr = Qr + kT * kP;      // [r][d]
  float* Ps = dOr + kT * kP;      // [r][c]
  float* dSs = Ps + kT * kP;      // [r][c]
  float* s_lse = dSs + kT * kP;   // [r]
  float* s_dv = s_lse + kT;       // [r]
  const int b = blockIdx.z, kvh = blockIdx.y, j0 = blockIdx.x * kT;
  const int g = a.H / a.KVH;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  load_tile(k, b, kvh, j0, a.L, a.D, 1.0f, Kt, nullptr);
  load_tile(v, b, kvh, j0, a.L, a.D, 1.0f, Vt, nullptr);
  float acc_dk[4][4] = {}, acc_dv[4][4] = {};
  int istart = 0;
  if (a.causal) {
    int first = j0 - a.pos_offset;
    istart = first > 0 ? (first / kT) * kT : 0;
  }
  for (int gi = 0; gi < g; gi++) {
    int h = kvh * g + gi;
    for (int i0 = istart; i0 < a.S; i0 += kT) {
      __syncthreads();
      load_tile(q, b, h, i0, a.S, a.D, a.scale, Qt, Qr);
      // dout is [B,S,H,D]: its row index is axis 1, so it is loaded here rather than through load_tile.
      for (int idx = threadIdx.x; idx < kT * kMaxD; idx += blockDim.x) {
        int r = idx / kMaxD, d = idx % kMaxD;
        float x = (i0 + r < a.S && d < a.D) ? dout.at(b, i0 + r, h, d) : 0.0f;
        dOt[d * kP + r] = x;
        dOr[r * kP + d] = x;
      }
      if (threadIdx.x < kT) {
        int r = i0 + threadIdx.x;
        s_lse[threadIdx.x] = r < a.S ? lse[((int64_t)b * a.H + h) * a.S + r] : 0.0f;
        s_dv[threadIdx.x] = r < a.S ? dvec[((int64_t)b * a.H + h) * a.S + r] : 0.0f;
      }
      __syncthreads();
      float s[4][4], dp[4][4];
      tile_dot(Qt, Kt, a.D, ty, tx, s);
      tile_dot(dOt, Vt, a.D, ty, tx, dp);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        int r = 4 * ty + i, qi = i0 + r;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          int c = 4 * tx + j;
          bool ok = qi < a.S && visible(a, qi, j0 + c);
          float p = ok ? expf(s[i][j] - s_lse[r]) : 0.0f;
          Ps[r * kP + c] = p;
          dSs[r * kP + c] = p * (dp[i][j] - s_dv[r]);
        }
      }
      __syncthreads();
      tile_acc(Ps, dOr, acc_dv);   // dV[c][d] += Σ_r P[r][c]·dO[r][d]
      tile_acc(dSs, Qr, acc_dk);   // dK[c][d] += Σ_r dS[r][c]·(q·scale)[r][d]
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int c = j0 + 4 * ty + i;
    if (c >= a.L) continue;
    int64_t base = (((int64_t)b * a.KVH + kvh) * a.L + c) * a.D;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int d = 4 * tx + j;
      if (d < a.D) { dk[base + d] = acc_dk[i][j]; dvv[base + d] = acc_dv[i][j]; }
    }
  }
}

// dQ for one 64-query tile of one head: Σ over visible key tiles, then × scale (the Mul(q, 1/√dh) rule).
__global__ void __launch_bounds__(256) k_attn_bwd_q(AttnDims a, V4 q, V4 k, V4 v, V4 dout, const float* __restrict__ lse,
                                                    const float* __restrict__ dvec, float* __restrict__ dq) {
  extern __shared__ float sm[];
  float* Qt = sm;                 // [d][r]
  float* dOt = Qt + kMaxD * kP;   // [d][r]
  float* Kt = dOt + kMaxD * kP;   // [d][c]
  float* Vt = Kt + kMaxD * kP;    // [d][c]
  float* Kr = Vt + kMaxD * kP;    // [c][d]
  float* dSt = Kr + kT * kP;      // [c][r]
  float* s_lse = dSt + kT * kP;
  float* s_dv = s_lse + kT;
  const int b = blockIdx.z, h = blockIdx.y, i0 = blockIdx.x * kT;
  const int kvh = h / (a.H / a.KVH);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  load_tile(q, b, h, i0, a.S, a.D, a.scale, Qt, nullptr);
  for (int idx = threadIdx.x; idx < kT * kMaxD; idx += blockDim.x) {
    int r = idx / kMaxD, d = idx % kMaxD;
    dOt[d * kP + r] = (i0 + r < a.S && d < a.D) ? dout.at(b, i0 + r, h, d) : 0.0f;
  }
  if (threadIdx.x < kT) {
    int r = i0 + threadIdx.x;
    s_lse[threadIdx.x] = r < a.S ? lse[((int64_t)b * a.H + h) * a.S + r] : 0.0f;
    s_dv[threadIdx.x] = r < a.S ? dvec[((int64_t)b * a.H + h) * a.S + r] : 0.0f;
  }
  float acc[4][4] = {};
  int kend = a.L;
  if (a.causal) kend = min(a.L, a.pos_offset + i0 + kT);
  for (int k0 = 0; k0 < kend; k0 += kT) {
    __syncthreads();
    load_tile(k, b, kvh, k0, a.L, a.D, 1.0f, Kt, Kr);
    load_tile(v, b, kvh, k0, a.L, a.D, 1.0f, Vt, nullptr);
    __syncthreads();
    float s[4][4], dp[4][4];
    tile_dot(Qt, Kt, a.D, ty, tx, s);
    tile_dot(dOt, Vt, a.D, ty, tx, dp);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      int r = 4 * ty + i, qi = i0 + r;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        int c = 4 * tx + j;
        bool ok = qi < a.S && visible(a, qi, k0 + c);
        float p = ok ? expf(s[i][j] - s_lse[r]) : 0.0f;
        dSt[c * kP + r] = p * (dp[i][j] - s_dv[r]);
      }
    }
    __syncthreads();
    tile_acc(dSt, Kr, acc);  // dQs[r][d] += Σ_c dS[r][c]·K[c][d]
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int qi = i0 + 4 * ty + i;
    if (qi >= a.S) continue;
    int64_t base = (((int64_t)b * a.H + h) * a.S + qi) * a.D;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int d = 4 * tx + j;
      if (d < a.D) dq[base + d] = acc[i][j] * a.scale;
    }
  }
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

constexpr size_t kFwdSmem = (size_t)(2 * kMaxD * kP + 2 * kT * kP) * 4;
constexpr size_t kKvSmem = (size_t)(4 * kMaxD * kP + 4 * kT * kP + 2 * kT) * 4;
constexpr size_t kQSmem = (size_t)(4 * kMaxD * kP + 2 * kT * kP + 2 * kT) * 4;

// PAI_ATTN=simt selects the CUDA-core kernels (used to cross-check the tensor-core path).
static bool attn_force_simt() {
  static int v = [] {
    const char* e = getenv("PAI_ATTN");
    return (e && strcmp(e, "simt") == 0) ? 1 : 0;
  }();
  return v != 0;
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
  if (numel(ro) > 0 && a.L > 0 && !attn_force_simt() && attn_decode_fits(*q, *k, *v, a.H, a.KVH, a.S, a.D)) {
    // decode step: HBM-bound split-KV kernel (attention_decode.cu); work = K and V bytes read
    int kend = causal ? std::min(a.L, pos_offset + a.S) : a.L;
    KernelTimerScope timer(ctx, "attn_decode", 8.0 * a.B * a.KVH * (double)kend * a.D);
    PAI_TRY(attn_decode_fwd(ctx, *q, *k, *v, a.B, a.H, a.KVH, a.S, a.L, a.D, scale, causal, pos_offset, fptr(ro), fptr(rl)));
  } else if (numel(ro) > 0 && a.L > 0) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_attn_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFwdSmem); attr = true; }
    KernelTimerScope timer(ctx, "attn_fwd", attn_fwd_flops(a));
    if (!attn_force_simt()) {
      PAI_TRY(attn_tc_fwd(ctx, *q, *k, *v, a.B, a.H, a.KVH, a.S, a.L, a.D, scale, causal, pos_offset, fptr(ro), fptr(rl)));
    } else {
      dim3 grid((unsigned)((a.S + kT - 1) / kT), (unsigned)a.H, (unsigned)a.B);
      k_attn_fwd<<<grid, 256, kFwdSmem, ctx->stream>>>(a, v4(*q), v4(*k), v4(*v), fptr(ro), fptr(rl));
      PAI_LAUNCH_CHECK("sdpa_fwd");
    }
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
  // the tensor-core kernels write every element of dq, dk and dv; the CUDA-core kernels and empty key ranges start
  // from zeros
  const bool zero = attn_force_simt() || a.L == 0;
  PAI_TRY(alloc_tensor(ctx, 4, qd, q->dtype, zero, &rq));
  PAI_TRY(alloc_tensor(ctx, 4, kd, q->dtype, zero, &rk));
  PAI_TRY(alloc_tensor(ctx, 4, kd, q->dtype, zero, &rv));
  if (numel(rq) > 0 && a.L > 0) {
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(k_attn_bwd_kv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kKvSmem);
      cudaFuncSetAttribute(k_attn_bwd_q, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kQSmem);
      attr = true;
    }
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
    if (!attn_force_simt()) {
      PAI_TRY(attn_tc_bwd(ctx, *q, *k, *v, *dout, fptr(*lse), static_cast<float*>(dvec.p), a.B, a.H, a.KVH, a.S, a.L, a.D,
                          scale, causal, pos_offset, fptr(rq), fptr(rk), fptr(rv)));
    } else {
      dim3 gkv((unsigned)((a.L + kT - 1) / kT), (unsigned)a.KVH, (unsigned)a.B);
      k_attn_bwd_kv<<<gkv, 256, kKvSmem, ctx->stream>>>(a, v4(*q), v4(*k), v4(*v), v4(*dout), fptr(*lse),
                                                        static_cast<float*>(dvec.p), fptr(rk), fptr(rv));
      PAI_LAUNCH_CHECK("sdpa_bwd kv");
      dim3 gq((unsigned)((a.S + kT - 1) / kT), (unsigned)a.H, (unsigned)a.B);
      k_attn_bwd_q<<<gq, 256, kQSmem, ctx->stream>>>(a, v4(*q), v4(*k), v4(*v), v4(*dout), fptr(*lse),
                                                     static_cast<float*>(dvec.p), fptr(rq));
      PAI_LAUNCH_CHECK("sdpa_bwd q");
    }
  }
  *dq = rq;
  *dk = rk;
  *dv = rv;
  return PAI_OK;
}
