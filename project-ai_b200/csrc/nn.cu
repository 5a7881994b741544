// RMSNorm, rotary embedding and the SwiGLU gate: HBM-streaming row kernels.
// Forward semantics: CpuComputeBackend.cs:361-382 (RmsNorm), :397-420 (RotaryEmbedding), :385-391 (Silu).
// Fused backward rules restate Autograd.cs:223-244 (RmsNorm) and :208-217 with the Mul rule (:39-47) for SwiGLU.
#include "common.cuh"

namespace pai {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float sigmoid_dev(float v) {
  if (v >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
  float t = expf(v);
  return __fdiv_rn(t, __fadd_rn(1.0f, t));
}

// ---------------------------------------------------------------- RMSNorm forward: one warp per row.
__global__ void k_rmsnorm_fwd(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                              int64_t rows, int d, float eps) {
  pdl_trigger();
  pdl_wait();
  int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const float* p = x + r * d;
    float ss = 0.0f;
    for (int j = lane; j < d; j += 32) { float v = p[j]; ss = fmaf(v, v, ss); }
    ss = warp_sum(ss);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
    float* q = y + r * d;
    for (int j = lane; j < d; j += 32) q[j] = __fmul_rn(__fmul_rn(p[j], inv), w[j]);
  }
}

// Rows of d = 128·C elements: each lane holds C float4 of the row, all loads issued before the reduction, so a warp
// needs one memory round trip per row instead of d/32 dependent loads (the decode case is a single row).
template <int C>
__global__ void __launch_bounds__(256) k_rmsnorm_fwd_reg(const float* __restrict__ x, const float* __restrict__ w,
                                                         float* __restrict__ y, int64_t rows, float eps) {
  constexpr int d = 128 * C;
  const int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  pdl_trigger();
  pdl_wait();
  for (int64_t r = warp; r < rows; r += nwarps) {
    const float4* px = reinterpret_cast<const float4*>(x + r * d);
    float4 xv[C];
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < C; c++) xv[c] = px[c * 32 + lane];
#pragma unroll
    for (int c = 0; c < C; c++) {
      ss = fmaf(xv[c].x, xv[c].x, ss); ss = fmaf(xv[c].y, xv[c].y, ss);
      ss = fmaf(xv[c].z, xv[c].z, ss); ss = fmaf(xv[c].w, xv[c].w, ss);
    }
    ss = warp_sum(ss);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
    float4* py = reinterpret_cast<float4*>(y + r * d);
#pragma unroll
    for (int c = 0; c < C; c++) {
      float4 wv = reinterpret_cast<const float4*>(w)[c * 32 + lane];
      float4 o;
      o.x = __fmul_rn(__fmul_rn(xv[c].x, inv), wv.x);
      o.y = __fmul_rn(__fmul_rn(xv[c].y, inv), wv.y);
      o.z = __fmul_rn(__fmul_rn(xv[c].z, inv), wv.z);
      o.w = __fmul_rn(__fmul_rn(xv[c].w, inv), wv.w);
      py[c * 32 + lane] = o;
    }
  }
}

// ---------------------------------------------------------------- RMSNorm backward.
// dx = inv·(g⊙w) − (inv²/D)·x·Σ(g⊙y);  dw partial per block = Σ_rows g⊙x·inv, reduced by k_colsum.
__global__ void k_rmsnorm_bwd(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ g,
                              float* __restrict__ dx, float* __restrict__ dw_part, int64_t rows, int d, float eps,
                              int rows_per_block) {
  extern __shared__ float s_dw[];  // [warps][d]
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float* my_dw = s_dw + (size_t)wid * d;
  for (int j = lane; j < d; j += 32) my_dw[j] = 0.0f;
  int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
  int64_t r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  for (int64_t r = r0 + wid; r < r1; r += nw) {
    const float* px = x + r * d;
    const float* pg = g + r * d;
    float ss = 0.0f;
    for (int j = lane; j < d; j += 32) { float v = px[j]; ss = fmaf(v, v, ss); }
    ss = warp_sum(ss);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
    float dot = 0.0f;
    for (int j = lane; j < d; j += 32) dot = fmaf(pg[j], px[j] * inv * w[j], dot);
    dot = warp_sum(dot);
    float coef = inv * inv / (float)d;
    float* pdx = dx + r * d;
    for (int j = lane; j < d; j += 32) {
      float gv = pg[j], xv = px[j];
      pdx[j] = (gv * w[j]) * inv - (coef * xv) * dot;
      my_dw[j] += gv * (xv * inv);
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float acc = 0.0f;
    for (int k = 0; k < nw; k++) acc += s_dw[(size_t)k * d + j];
    dw_part[(size_t)blockIdx.x * d + j] = acc;
  }
}

// The same rule with each row held in registers (d = 128·C): one read of x and g, dx written once, and each lane
// accumulating its own columns of dw across the rows its warp visits; partials reduced per block in shared memory.
// Rows longer than 1024 (C > 8) keep the dw partials in the warp's shared-memory row and read w through the
// read-only cache instead of holding both in registers (x, g, w and the partials at C = 16 would need ~256
// registers and spill); the per-element operations and their order are the same.
template <int C>
__global__ void __launch_bounds__(256) k_rmsnorm_bwd_reg(const float* __restrict__ x, const float* __restrict__ w,
                                                         const float* __restrict__ g, float* __restrict__ dx,
                                                         float* __restrict__ dw_part, int64_t rows, float eps) {
  extern __shared__ float s_dw[];  // [warps][d]
  constexpr int d = 128 * C;
  constexpr bool kSmemAcc = C > 8;
  constexpr int CR = kSmemAcc ? 1 : C;  // register-held w and dw partials
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float4* my_acc = reinterpret_cast<float4*>(s_dw + (size_t)wid * d);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 wv[CR], acc[CR];
#pragma unroll
  for (int c = 0; c < CR; c++) {
    wv[c] = kSmemAcc ? make_float4(0.f, 0.f, 0.f, 0.f) : w4[c * 32 + lane];
    acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (kSmemAcc) {
#pragma unroll
    for (int c = 0; c < C; c++) my_acc[c * 32 + lane] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int64_t r = (int64_t)blockIdx.x * nw + wid; r < rows; r += (int64_t)gridDim.x * nw) {
    const float4* px = reinterpret_cast<const float4*>(x + r * d);
    const float4* pg = reinterpret_cast<const float4*>(g + r * d);
    float4 xv[C], gv[C];
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < C; c++) {
      xv[c] = px[c * 32 + lane];
      gv[c] = pg[c * 32 + lane];
      ss = fmaf(xv[c].x, xv[c].x, ss); ss = fmaf(xv[c].y, xv[c].y, ss);
      ss = fmaf(xv[c].z, xv[c].z, ss); ss = fmaf(xv[c].w, xv[c].w, ss);
    }
    ss = warp_sum(ss);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
    float dot = 0.0f;
#pragma unroll
    for (int c = 0; c < C; c++) {
      const float4 wc = kSmemAcc ? __ldg(w4 + c * 32 + lane) : wv[kSmemAcc ? 0 : c];
      dot = fmaf(gv[c].x, xv[c].x * inv * wc.x, dot); dot = fmaf(gv[c].y, xv[c].y * inv * wc.y, dot);
      dot = fmaf(gv[c].z, xv[c].z * inv * wc.z, dot); dot = fmaf(gv[c].w, xv[c].w * inv * wc.w, dot);
    }
    dot = warp_sum(dot);
    float coef = inv * inv / (float)d;
    float4* pdx = reinterpret_cast<float4*>(dx + r * d);
#pragma unroll
    for (int c = 0; c < C; c++) {
      const float4 wc = kSmemAcc ? __ldg(w4 + c * 32 + lane) : wv[kSmemAcc ? 0 : c];
      float4 o;
      o.x = (gv[c].x * wc.x) * inv - (coef * xv[c].x) * dot;
      o.y = (gv[c].y * wc.y) * inv - (coef * xv[c].y) * dot;
      o.z = (gv[c].z * wc.z) * inv - (coef * xv[c].z) * dot;
      o.w = (gv[c].w * wc.w) * inv - (coef * xv[c].w) * dot;
      pdx[c * 32 + lane] = o;
      float4 a = kSmemAcc ? my_acc[c * 32 + lane] : acc[kSmemAcc ? 0 : c];
      a.x += gv[c].x * (xv[c].x * inv); a.y += gv[c].y * (xv[c].y * inv);
      a.z += gv[c].z * (xv[c].z * inv); a.w += gv[c].w * (xv[c].w * inv);
      if (kSmemAcc) my_acc[c * 32 + lane] = a;
      else acc[kSmemAcc ? 0 : c] = a;
    }
  }
  if (!kSmemAcc) {
#pragma unroll
    for (int c = 0; c < CR; c++) my_acc[c * 32 + lane] = acc[c];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float s = 0.0f;
    for (int k = 0; k < nw; k++) s += s_dw[(size_t)k * d + j];
    dw_part[(size_t)blockIdx.x * d + j] = s;
  }
}

// Deterministic column sum of [parts, d] partials with more loads in flight: a CTA takes 32 columns, its 8 warps each
// add a contiguous slice of the parts in order, and the 8 slice sums are added in slice order. Launch: (d + 31) / 32
// CTAs of 256 threads.
__global__ void __launch_bounds__(256) k_colsum_sliced(const float* __restrict__ part, float* __restrict__ out, int parts,
                                                       int d) {
  __shared__ float s[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  const int per = (parts + 7) / 8;
  const int p0 = w * per, p1 = min(parts, p0 + per);
  float acc = 0.0f;
  if (j < d) {
#pragma unroll 4
    for (int p = p0; p < p1; p++) acc += part[(size_t)p * d + j];
  }
  s[w][lane] = acc;
  __syncthreads();
  if (w == 0 && j < d) {
    float t = s[0][lane];
    for (int k = 1; k < 8; k++) t += s[k][lane];
    out[j] = t;
  }
}

// Deterministic column sum of [parts, d] partials.
__global__ void k_colsum(const float* __restrict__ part, float* __restrict__ out, int parts, int d) {
  int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d) return;
  float acc = 0.0f;
  for (int p = 0; p < parts; p++) acc += part[(size_t)p * d + j];
  out[j] = acc;
}

// ---------------------------------------------------------------- RoPE (rotate-half), generic views.
__global__ void k_rotary(const float* __restrict__ x, DView xv, const float* __restrict__ cs, DView cv,
                         const float* __restrict__ sn, DView sv, float* __restrict__ y, int64_t pairs, int d) {
  int half = d >> 1;
  for (int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; id < pairs; id += (int64_t)gridDim.x * blockDim.x) {
    int64_t row = id / half;
    int j = (int)(id - row * half);
    int64_t i0 = row * d + j, i1 = i0 + half;
    float x0 = x[dview_offset(xv, i0)], x1 = x[dview_offset(xv, i1)];
    float c0 = cs[dview_offset(cv, i0)], c1 = cs[dview_offset(cv, i1)];
    float s0 = sn[dview_offset(sv, i0)], s1 = sn[dview_offset(sv, i1)];
    // y[i] = x[i]·cos[i] + rot[i]·sin[i], rot = (−x[i+half], x[i−half])
    y[i0] = __fadd_rn(__fmul_rn(x0, c0), __fmul_rn(-x1, s0));
    y[i1] = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1));
  }
}

// Row-wise RoPE when the head dim is unit-stride in x, cos and sin: one warp per row, the row's offsets computed
// once from the leading dims, the row itself read and written contiguously.
// RopeShift: optional position read on the device (pai_rotary_at). The cos/sin views address table rows 0..S-1;
// the kernel moves them down by pos rows, after checking pos + S <= table_rows.
struct RopeShift {
  const float* pos = nullptr;
  int64_t stride_c = 0, stride_s = 0;  // element stride of one table row
  int seq = 0, table_rows = 0;
  int* error_flag = nullptr;
};

__global__ void k_rotary_rows(const float* __restrict__ x, DView xr, const float* __restrict__ cs, DView cr,
                              const float* __restrict__ sn, DView sr, float* __restrict__ y, int64_t rows, int d,
                              RopeShift shift) {
  int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int half = d >> 1;
  int64_t dc = 0, ds = 0;
  if (shift.pos) {
    float pf = shift.pos[0];
    int p = (int)pf;
    if (!(pf >= 0.0f) || p + shift.seq > shift.table_rows) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(shift.error_flag, 61);
      return;
    }
    dc = (int64_t)p * shift.stride_c;
    ds = (int64_t)p * shift.stride_s;
  }
  for (int64_t r = warp; r < rows; r += nwarps) {
    int64_t xo, co, so;
    row_offsets3(xr, cr, sr, (uint32_t)r, xo, co, so);
    co += dc;
    so += ds;
    float* yr = y + r * d;
    for (int j = lane; j < half; j += 32) {
      float x0 = x[xo + j], x1 = x[xo + j + half];
      yr[j] = __fadd_rn(__fmul_rn(x0, cs[co + j]), __fmul_rn(-x1, sn[so + j]));
      yr[j + half] = __fadd_rn(__fmul_rn(x1, cs[co + j + half]), __fmul_rn(x0, sn[so + j + half]));
    }
  }
}

// k_rotary_rows with one thread per 4 consecutive pairs (j..j+3, j+h..j+h+3) of a row: 16-byte loads of x, cos and
// sin and 16-byte stores, all independent, so the pass streams at memory speed. Needs d % 8 == 0 and every row
// start of x, cos and sin 16-byte aligned; the same element operations as k_rotary_rows.
// HQ: float4 groups per half row when it is a compile-time constant (head dim 64: 8), else 0 (runtime d >> 3). Item
// indices run in 32 bits when they fit (the integer division per item is the kernel's main instruction cost).
template <int HQ, typename Idx>
__global__ void k_rotary_rows4(const float* __restrict__ x, DView xr, const float* __restrict__ cs, DView cr,
                               const float* __restrict__ sn, DView sr, float* __restrict__ y, int64_t rows, int d,
                               RopeShift shift) {
  const int hq = HQ ? HQ : d >> 3;
  const int half = 4 * hq;
  int64_t dc = 0, ds = 0;
  if (shift.pos) {
    float pf = shift.pos[0];
    int p = (int)pf;
    if (!(pf >= 0.0f) || p + shift.seq > shift.table_rows) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(shift.error_flag, 61);
      return;
    }
    dc = (int64_t)p * shift.stride_c;
    ds = (int64_t)p * shift.stride_s;
  }
  const Idx total = (Idx)(rows * hq);
  for (Idx i = blockIdx.x * (Idx)blockDim.x + threadIdx.x; i < total; i += (Idx)gridDim.x * blockDim.x) {
    const Idx r = i / (Idx)hq;
    const int j = (int)(i - r * (Idx)hq) * 4;
    int64_t xo, co, so;
    row_offsets3(xr, cr, sr, (uint32_t)r, xo, co, so);
    co += dc;
    so += ds;
    const float4 x0 = *reinterpret_cast<const float4*>(x + xo + j), x1 = *reinterpret_cast<const float4*>(x + xo + j + half);
    const float4 c0 = *reinterpret_cast<const float4*>(cs + co + j), c1 = *reinterpret_cast<const float4*>(cs + co + j + half);
    const float4 s0 = *reinterpret_cast<const float4*>(sn + so + j), s1 = *reinterpret_cast<const float4*>(sn + so + j + half);
    float4 y0, y1;
    y0.x = __fadd_rn(__fmul_rn(x0.x, c0.x), __fmul_rn(-x1.x, s0.x));
    y0.y = __fadd_rn(__fmul_rn(x0.y, c0.y), __fmul_rn(-x1.y, s0.y));
    y0.z = __fadd_rn(__fmul_rn(x0.z, c0.z), __fmul_rn(-x1.z, s0.z));
    y0.w = __fadd_rn(__fmul_rn(x0.w, c0.w), __fmul_rn(-x1.w, s0.w));
    y1.x = __fadd_rn(__fmul_rn(x1.x, c1.x), __fmul_rn(x0.x, s1.x));
    y1.y = __fadd_rn(__fmul_rn(x1.y, c1.y), __fmul_rn(x0.y, s1.y));
    y1.z = __fadd_rn(__fmul_rn(x1.z, c1.z), __fmul_rn(x0.z, s1.z));
    y1.w = __fadd_rn(__fmul_rn(x1.w, c1.w), __fmul_rn(x0.w, s1.w));
    float* yr = y + r * d;
    *reinterpret_cast<float4*>(yr + j) = y0;
    *reinterpret_cast<float4*>(yr + j + half) = y1;
  }
}

// ---------------------------------------------------------------- SwiGLU gate
__device__ __forceinline__ float silu_mul_elem(float gv, float u) { return silu_mul_value(gv, u); }

__device__ __forceinline__ void silu_mul_bwd_elem(float gv, float u, float go, float& dg, float& du) {
  float s = sigmoid_dev(gv);
  float y = __fmul_rn(gv, s);
  float dsilu = __fmul_rn(go, u);                               // Mul rule: d(silu) = g·up
  du = __fmul_rn(go, y);                                         //           d(up)   = g·silu
  float deriv = __fsub_rn(__fadd_rn(s, y), __fmul_rn(s, y));      // Silu rule: s + y − s·y
  dg = __fmul_rn(dsilu, deriv);
}

// n4 = number of float4 groups; the scalar tail [4*n4, n) is handled by the same grid.
__global__ void k_silu_mul_fwd(const float* __restrict__ gate, const float* __restrict__ up, float* __restrict__ o,
                               int64_t n, bool vec) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  int64_t n4 = vec ? n >> 2 : 0;
  // two float4 of each input per trip: four 16-byte loads in flight per thread before the first store
  for (int64_t i = tid; i < n4; i += 2 * stride) {
    const int64_t i2 = i + stride;
    const bool two = i2 < n4;
    float4 g4 = reinterpret_cast<const float4*>(gate)[i], u4 = reinterpret_cast<const float4*>(up)[i];
    float4 g5 = two ? reinterpret_cast<const float4*>(gate)[i2] : g4, u5 = two ? reinterpret_cast<const float4*>(up)[i2] : u4;
    reinterpret_cast<float4*>(o)[i] =
        make_float4(silu_mul_elem(g4.x, u4.x), silu_mul_elem(g4.y, u4.y), silu_mul_elem(g4.z, u4.z), silu_mul_elem(g4.w, u4.w));
    if (two)
      reinterpret_cast<float4*>(o)[i2] =
          make_float4(silu_mul_elem(g5.x, u5.x), silu_mul_elem(g5.y, u5.y), silu_mul_elem(g5.z, u5.z), silu_mul_elem(g5.w, u5.w));
  }
  for (int64_t i = (n4 << 2) + tid; i < n; i += stride) o[i] = silu_mul_elem(gate[i], up[i]);
}

__global__ void k_silu_mul_bwd(const float* __restrict__ gate, const float* __restrict__ up, const float* __restrict__ g,
                               float* __restrict__ dgate, float* __restrict__ dup, int64_t n, bool vec) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  int64_t n4 = vec ? n >> 2 : 0;
  for (int64_t i = tid; i < n4; i += stride) {
    float4 g4 = reinterpret_cast<const float4*>(gate)[i], u4 = reinterpret_cast<const float4*>(up)[i];
    float4 o4 = reinterpret_cast<const float4*>(g)[i];
    float4 dg, du;
    silu_mul_bwd_elem(g4.x, u4.x, o4.x, dg.x, du.x);
    silu_mul_bwd_elem(g4.y, u4.y, o4.y, dg.y, du.y);
    silu_mul_bwd_elem(g4.z, u4.z, o4.z, dg.z, du.z);
    silu_mul_bwd_elem(g4.w, u4.w, o4.w, dg.w, du.w);
    reinterpret_cast<float4*>(dgate)[i] = dg;
    reinterpret_cast<float4*>(dup)[i] = du;
  }
  for (int64_t i = (n4 << 2) + tid; i < n; i += stride) silu_mul_bwd_elem(gate[i], up[i], g[i], dgate[i], dup[i]);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_rmsnorm(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* w, float eps, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  PAI_TRY(check_view(ctx, w, "weight"));
  if (x->rank == 0) return set_error(PAI_ERR_ARGUMENT, "RmsNorm requires rank >= 1.");
  int d = x->dims[x->rank - 1];
  if (w->rank != 1 || w->dims[0] != d)
    return set_error(PAI_ERR_ARGUMENT, "RmsNorm weight must be [%d] to match the last axis of %s.", d, shape_str(*x).c_str());
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, x->rank, x->dims, x->dtype, false, &r));
  int64_t rows = d ? numel(*x) / d : 0;
  if (rows > 0) {
    const float *xp, *wp;
    Scratch hx, hw;
    PAI_TRY(dense_input(ctx, *x, &xp, &hx));
    PAI_TRY(dense_input(ctx, *w, &wp, &hw));
    int chunks = d % 128 == 0 ? d / 128 : 0;
    bool aligned = aligned16(xp) && aligned16(wp) && aligned16(fptr(r));
    int grid = grid_for(ctx, rows * 32, 256);
    float* yp = fptr(r);
    cudaError_t e;
    dim3 g(grid), blk(256);
    switch (aligned ? chunks : 0) {
      case 1: e = launch_pdl(k_rmsnorm_fwd_reg<1>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      case 2: e = launch_pdl(k_rmsnorm_fwd_reg<2>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      case 4: e = launch_pdl(k_rmsnorm_fwd_reg<4>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      case 6: e = launch_pdl(k_rmsnorm_fwd_reg<6>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      case 8: e = launch_pdl(k_rmsnorm_fwd_reg<8>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      case 12: e = launch_pdl(k_rmsnorm_fwd_reg<12>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      case 16: e = launch_pdl(k_rmsnorm_fwd_reg<16>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      case 32: e = launch_pdl(k_rmsnorm_fwd_reg<32>, g, blk, 0, ctx->stream, xp, wp, yp, rows, eps); break;
      default: e = launch_pdl(k_rmsnorm_fwd, g, blk, 0, ctx->stream, xp, wp, yp, rows, d, eps); break;
    }
    if (e != cudaSuccess) return cuda_error(e, "rmsnorm");
    ctx->launches++;
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_rmsnorm_bwd(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* w, const pai_tensor* g, float eps,
                                   pai_tensor* dx, pai_tensor* dw) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  PAI_TRY(check_view(ctx, w, "weight"));
  PAI_TRY(check_view(ctx, g, "grad"));
  if (x->rank == 0) return set_error(PAI_ERR_ARGUMENT, "RmsNorm requires rank >= 1.");
  int d = x->dims[x->rank - 1];
  if (w->rank != 1 || w->dims[0] != d || numel(*g) != numel(*x))
    return set_error(PAI_ERR_ARGUMENT, "RmsNormBackward: shapes disagree (%s, %s, %s)", shape_str(*x).c_str(),
                     shape_str(*w).c_str(), shape_str(*g).c_str());
  pai_tensor rdx, rdw;
  int64_t rows = d ? numel(*x) / d : 0;
  PAI_TRY(alloc_tensor(ctx, x->rank, x->dims, x->dtype, false, &rdx));
  PAI_TRY(alloc_tensor(ctx, 1, &d, x->dtype, rows == 0, &rdw));  // the column sum writes every entry
  if (rows > 0) {
    const float *xp, *wp, *gp;
    Scratch hx, hw, hg, part;
    PAI_TRY(dense_input(ctx, *x, &xp, &hx));
    PAI_TRY(dense_input(ctx, *w, &wp, &hw));
    PAI_TRY(dense_input(ctx, *g, &gp, &hg));
    bool aligned = aligned16(xp) && aligned16(wp) && aligned16(gp) && aligned16(fptr(rdx));
    int chunks = d % 128 == 0 ? d / 128 : 0;
    if (aligned && (chunks == 1 || chunks == 2 || chunks == 4 || chunks == 6 || chunks == 8 || chunks == 16)) {
      int blocks = (int)std::min<int64_t>(ctx->sm_count, (rows + 7) / 8);
      size_t smem = (size_t)8 * d * 4;
      PAI_TRY(scratch(ctx, (size_t)blocks * d * 4, &part));
      float* pp = static_cast<float*>(part.p);
#define RMS_REG(C)                                                                                              \
  do {                                                                                                          \
    if (smem > 48 * 1024) PAI_CUDA(smem_limit(ctx, k_rmsnorm_bwd_reg<C>, (int)smem));                                  \
    k_rmsnorm_bwd_reg<C><<<blocks, 256, smem, ctx->stream>>>(xp, wp, gp, fptr(rdx), pp, rows, eps);            \
  } while (0)
      switch (chunks) {
        case 1: RMS_REG(1); break;
        case 2: RMS_REG(2); break;
        case 4: RMS_REG(4); break;
        case 6: RMS_REG(6); break;
        case 8: RMS_REG(8); break;
        default: RMS_REG(16); break;
      }
#undef RMS_REG
      PAI_LAUNCH_CHECK("rmsnorm_bwd");
      k_colsum_sliced<<<(d + 31) / 32, 256, 0, ctx->stream>>>(pp, fptr(rdw), blocks, d);
      PAI_LAUNCH_CHECK("rmsnorm_bwd colsum");
      *dx = rdx;
      *dw = rdw;
      return PAI_OK;
    }
    int threads = 256, nw = threads / 32;
    size_t smem = (size_t)nw * d * 4;
    if (smem > 200 * 1024) { threads = 64; nw = 2; smem = (size_t)nw * d * 4; }
    if (smem > 200 * 1024) return set_error(PAI_ERR_UNSUPPORTED, "RmsNormBackward: row length %d too large", d);
    int blocks = ctx->sm_count * 2;
    int rpb = (int)((rows + blocks - 1) / blocks);
    if (rpb < nw) rpb = nw;
    blocks = (int)((rows + rpb - 1) / rpb);
    PAI_TRY(scratch(ctx, (size_t)blocks * d * 4, &part));
    if (smem > 48 * 1024) PAI_CUDA(smem_limit(ctx, k_rmsnorm_bwd, (int)smem));
    k_rmsnorm_bwd<<<blocks, threads, smem, ctx->stream>>>(xp, wp, gp, fptr(rdx), static_cast<float*>(part.p), rows, d, eps, rpb);
    PAI_LAUNCH_CHECK("rmsnorm_bwd");
    k_colsum_sliced<<<(d + 31) / 32, 256, 0, ctx->stream>>>(static_cast<float*>(part.p), fptr(rdw), blocks, d);
    PAI_LAUNCH_CHECK("rmsnorm_bwd colsum");
  }
  *dx = rdx;
  *dw = rdw;
  return PAI_OK;
}

static pai_status rotary_impl(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* cs, const pai_tensor* sn,
                              const RopeShift& shift, pai_tensor* out);

PAI_API pai_status pai_rotary(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* cs, const pai_tensor* sn, pai_tensor* out) {
  return rotary_impl(ctx, x, cs, sn, RopeShift{}, out);
}

PAI_API pai_status pai_rotary_at(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* cos_table, const pai_tensor* sin_table,
                                 const pai_tensor* pos, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  PAI_TRY(check_view(ctx, cos_table, "cos"));
  PAI_TRY(check_view(ctx, sin_table, "sin"));
  PAI_TRY(check_view(ctx, pos, "pos"));
  if (x->rank < 2 || cos_table->rank != 2 || sin_table->rank != 2 || numel(*pos) != 1)
    return set_error(PAI_ERR_ARGUMENT, "RotaryAt: x [..., S, d], tables [T, d] and a one-element position expected");
  int seq = x->dims[x->rank - 2], d = x->dims[x->rank - 1];
  int rows = cos_table->dims[0];
  if (cos_table->dims[1] != d || sin_table->dims[1] != d || sin_table->dims[0] != rows || seq > rows)
    return set_error(PAI_ERR_ARGUMENT, "RotaryAt: tables %s / %s do not fit x %s", shape_str(*cos_table).c_str(),
                     shape_str(*sin_table).c_str(), shape_str(*x).c_str());
  if (x->strides[x->rank - 1] != 1 || cos_table->strides[1] != 1 || sin_table->strides[1] != 1)
    return set_error(PAI_ERR_UNSUPPORTED, "RotaryAt: rows must be contiguous");
  // table rows 0..S-1; the kernel adds pos rows
  pai_tensor c = *cos_table, sv = *sin_table;
  c.dims[0] = seq;
  sv.dims[0] = seq;
  RopeShift shift;
  shift.pos = fptr(*pos);
  shift.stride_c = cos_table->strides[0];
  shift.stride_s = sin_table->strides[0];
  shift.seq = seq;
  shift.table_rows = rows;
  shift.error_flag = ctx->d_error_flag;
  return rotary_impl(ctx, x, &c, &sv, shift, out);
}

static pai_status rotary_impl(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* cs, const pai_tensor* sn,
                              const RopeShift& shift, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  PAI_TRY(check_view(ctx, cs, "cos"));
  PAI_TRY(check_view(ctx, sn, "sin"));
  int rank = x->rank;
  if (rank == 0) return set_error(PAI_ERR_ARGUMENT, "RotaryEmbedding requires rank >= 1.");
  int d = x->dims[rank - 1];
  if (d % 2) return set_error(PAI_ERR_ARGUMENT, "RoPE head dim must be even; got %d.", d);
  auto ok = [&](const pai_tensor* t) {
    if (t->rank > rank) return false;
    int lead = rank - t->rank;
    for (int i = 0; i < t->rank; i++)
      if (t->dims[i] != x->dims[lead + i] && t->dims[i] != 1) return false;
    return true;
  };
  if (!ok(cs) || !ok(sn)) return set_error(PAI_ERR_ARGUMENT, "Cannot broadcast cos/sin to %s.", shape_str(*x).c_str());
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, rank, x->dims, x->dtype, false, &r));
  int64_t n = numel(*x);
  if (n > 0) {
    pai_tensor cb = broadcast_view(*cs, rank, x->dims), sb = broadcast_view(*sn, rank, x->dims);
    const pai_tensor* views[3] = {x, &cb, &sb};
    DView dv[3];
    bool unit_last = (x->strides[rank - 1] == 1 && cb.strides[rank - 1] == 1 && sb.strides[rank - 1] == 1) &&
                     n / d < (1ll << 31);
    if (unit_last) {
      collapse(rank - 1, x->dims, views, 3, dv);  // leading (row) dims only
      int64_t rows = n / d;
      // 16-byte path: every row start of x, cos and sin (any position shift included) on a 16-byte boundary
      bool vec4 = d % 8 == 0 && (shift.stride_c % 4 == 0) && (shift.stride_s % 4 == 0);
      const void* bases[3] = {x->base, cs->base, sn->base};
      for (int v = 0; v < 3 && vec4; v++) {
        if ((uintptr_t)bases[v] % 16 || dv[v].offset % 4) vec4 = false;
        for (int i = 0; i < dv[v].rank; i++)
          if (dv[v].dims[i] > 1 && dv[v].strides[i] % 4) vec4 = false;
      }
      if (vec4) {
        const dim3 g(grid_for(ctx, rows * (d / 8), 256));
        const bool small = rows * (d / 8) < (int64_t)INT32_MAX;
        const float *xb = static_cast<const float*>(x->base), *cb = static_cast<const float*>(cs->base),
                    *sb = static_cast<const float*>(sn->base);
        if (d == 64 && small) k_rotary_rows4<8, uint32_t><<<g, 256, 0, ctx->stream>>>(xb, dv[0], cb, dv[1], sb, dv[2], fptr(r), rows, d, shift);
        else if (small) k_rotary_rows4<0, uint32_t><<<g, 256, 0, ctx->stream>>>(xb, dv[0], cb, dv[1], sb, dv[2], fptr(r), rows, d, shift);
        else k_rotary_rows4<0, int64_t><<<g, 256, 0, ctx->stream>>>(xb, dv[0], cb, dv[1], sb, dv[2], fptr(r), rows, d, shift);
      } else {
        k_rotary_rows<<<grid_for(ctx, rows * 32, 256), 256, 0, ctx->stream>>>(
            static_cast<const float*>(x->base), dv[0], static_cast<const float*>(cs->base), dv[1],
            static_cast<const float*>(sn->base), dv[2], fptr(r), rows, d, shift);
      }
    } else if (shift.pos) {
      raw_free(ctx, r.base);
      return set_error(PAI_ERR_UNSUPPORTED, "RotaryAt: rows must be contiguous");
    } else {
      collapse(rank, x->dims, views, 3, dv);
      int64_t pairs = n / 2;
      k_rotary<<<grid_for(ctx, pairs, 256), 256, 0, ctx->stream>>>(static_cast<const float*>(x->base), dv[0],
                                                                 static_cast<const float*>(cs->base), dv[1],
                                                                 static_cast<const float*>(sn->base), dv[2], fptr(r), pairs, d);
    }
    PAI_LAUNCH_CHECK("rotary");
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_silu_mul_fwd(pai_ctx* ctx, const pai_tensor* gate, const pai_tensor* up, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, gate, "gate"));
  PAI_TRY(check_view(ctx, up, "up"));
  if (gate->rank != up->rank || numel(*gate) != numel(*up))
    return set_error(PAI_ERR_ARGUMENT, "SiluMul: shapes differ (%s vs %s)", shape_str(*gate).c_str(), shape_str(*up).c_str());
  for (int i = 0; i < gate->rank; i++)
    if (gate->dims[i] != up->dims[i]) return set_error(PAI_ERR_ARGUMENT, "SiluMul: shapes differ");
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, gate->rank, gate->dims, gate->dtype, false, &r));
  int64_t n = numel(r);
  if (n > 0) {
    const float *gp, *up_;
    Scratch h1, h2;
    PAI_TRY(dense_input(ctx, *gate, &gp, &h1));
    PAI_TRY(dense_input(ctx, *up, &up_, &h2));
    bool vec = aligned16(gp) && aligned16(up_) && aligned16(fptr(r));
    k_silu_mul_fwd<<<grid_for(ctx, n, 256, vec ? 4 : 1), 256, 0, ctx->stream>>>(gp, up_, fptr(r), n, vec);
    PAI_LAUNCH_CHECK("silu_mul_fwd");
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_silu_mul_bwd(pai_ctx* ctx, const pai_tensor* gate, const pai_tensor* up, const pai_tensor* g,
                                    pai_tensor* dgate, pai_tensor* dup) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, gate, "gate"));
  PAI_TRY(check_view(ctx, up, "up"));
  PAI_TRY(check_view(ctx, g, "grad"));
  int64_t n = numel(*gate);
  if (numel(*up) != n || numel(*g) != n) return set_error(PAI_ERR_ARGUMENT, "SiluMulBackward: shapes differ");
  pai_tensor r1, r2;
  PAI_TRY(alloc_tensor(ctx, gate->rank, gate->dims, gate->dtype, false, &r1));
  PAI_TRY(alloc_tensor(ctx, gate->rank, gate->dims, gate->dtype, false, &r2));
  if (n > 0) {
    const float *gp, *up_, *gg;
    Scratch h1, h2, h3;
    PAI_TRY(dense_input(ctx, *gate, &gp, &h1));
    PAI_TRY(dense_input(ctx, *up, &up_, &h2));
    PAI_TRY(dense_input(ctx, *g, &gg, &h3));
    bool vec = aligned16(gp) && aligned16(up_) && aligned16(gg) && aligned16(fptr(r1)) && aligned16(fptr(r2));
    k_silu_mul_bwd<<<grid_for(ctx, n, 256, vec ? 4 : 1), 256, 0, ctx->stream>>>(gp, up_, gg, fptr(r1), fptr(r2), n, vec);
    PAI_LAUNCH_CHECK("silu_mul_bwd");
  }
  *dgate = r1;
  *dup = r2;
  return PAI_OK;
}
