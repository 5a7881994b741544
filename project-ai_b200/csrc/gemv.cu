// Small-M products y = x · Wᵀ for decode (IComputeBackend.MatMul with transposeB, CpuComputeBackend.cs:159-219):
// at most 32 rows of x against one weight matrix W [n, k]. Such a product is bound by streaming W from HBM
// (2 flops per 4-byte weight and x row), so it runs as a weight-streaming kernel in exact fp32 FMA arithmetic instead of
// the 128-row tensor-core tiles, which would pack W (read once, write hi+lo) and then read hi+lo again.
//
// Layout: each warp owns 4 consecutive W rows; its lanes stride K in 16-byte chunks (one coalesced 512-byte load per
// row per warp step, evict-first so the weights do not displace x from L1/L2). Every W chunk is multiplied against
// all rows of x (x is tiny and stays cached). When n is small, the warps of one CTA split K for the same 4 rows and
// their partial sums are added in warp order through shared memory, so results are deterministic run to run.
//
// From 5 to 32 rows the FMA work (2·rows flops per weight) outgrows the CUDA cores, so those products run on the
// tensor cores with the roles swapped (k_gemv_tc): yᵀ[n, rows] = W[n, :] · xᵀ, W supplying the 128-row A operand and
// x the 16- or 32-column B operand, in 3xTF32 (hi·hi + hi·lo + lo·hi, as in gemm.cu). W still crosses HBM once,
// in fp32: TMA brings each 128 x 32 fp32 W tile into shared memory (SWIZZLE_128B), four converter warps split it
// into tf32 hi/lo and store both into tensor memory, and the MMA reads A from tensor memory (tcgen05.mma [a_tmem]).
// x is split once per call into pre-swizzled hi/lo tiles that the producer bulk-copies beside each W tile.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace pai {

constexpr int kGemvMaxRows = 32;
constexpr int kGemvRowsPerWarp = 4;
constexpr int kGemvThreads = 256;

constexpr int kGemvMaxSegs = 4;
constexpr int kGemvTcMinRows = 5;  // from 5 rows of x the products run on the tensor cores

// Output epilogues: plain store, residual + x·Wᵀ (TransformerBlock's Add after a Linear), and SiLU(x·W0ᵀ)·(x·W1ᵀ)
// (SwiGLU's gate and up products combined as SiluMul does).
enum GemvMode { kGemvStore = 0, kGemvResidual = 1, kGemvSiluMul = 2 };

struct GemvArgs {
  // logical output columns [seg_start[s], seg_start[s+1]) come from rows of w[s] (row stride sw[s], unit column stride);
  // in SiLU·mul mode segment 0 is the gate and segment 1 the up projection, over the same columns
  const float* w[kGemvMaxSegs];
  int64_t sw[kGemvMaxSegs];
  int seg_start[kGemvMaxSegs + 1];
  int nseg;
  const float* x;                // base of x
  int64_t xoff[kGemvMaxRows];    // element offset of each x row (contiguous along k)
  float* y;                      // output row m at y + m * ldy
  int64_t ldy;
  const float* res;              // residual row m at res + m * ldr (residual mode)
  int64_t ldr;
  int rows, n, k;                // n = logical output columns
  int ksplit;                    // warps that share one group of 4 W rows (1, 2, 4 or 8)
  int mode;
  const float* norm_w;           // when set, x rows are RMS-normalised with this weight before the product
  float eps;
};

// 1 / sqrt(mean(x²) + eps) of one row of k elements, summed as k_rmsnorm_fwd_reg does for k = 128·C (lane-interleaved
// float4 chunks, then a warp sum) and as k_rmsnorm_fwd does otherwise, so the normalised row is bit-identical to the
// separate RmsNorm kernel's output.
__device__ __forceinline__ float row_inv_rms(const float* x, int k, float eps, bool vec) {
  const int lane = threadIdx.x & 31;
  float ss = 0.0f;
  if (vec && k % 128 == 0) {
    for (int c = 0; c < k / 128; c++) {
      float4 v = reinterpret_cast<const float4*>(x)[c * 32 + lane];
      ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
    }
  } else {
    for (int j = lane; j < k; j += 32) { float v = x[j]; ss = fmaf(v, v, ss); }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)k), eps)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void gemv_store(const GemvArgs& a, int m, int col, float v0, float v1) {
  float out = v0;
  if (a.mode == kGemvResidual) out = __fadd_rn(a.res[(int64_t)m * a.ldr + col], v0);
  else if (a.mode == kGemvSiluMul) out = silu_mul_value(v0, v1);
  a.y[(int64_t)m * a.ldy + col] = out;
}

// P = 1: each warp owns 4 logical columns (rows of their segment's W); P = 2 (SiLU·mul): the same 4 rows of both W.
template <int MR, int U, bool VEC, int P>
__global__ void __launch_bounds__(kGemvThreads) k_gemv_tn(const GemvArgs a) {
  constexpr int R = kGemvRowsPerWarp;
  constexpr int kWarps = kGemvThreads / 32;
  __shared__ float part[kWarps][MR][P][R];
  __shared__ float s_inv[MR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups_per_cta = kWarps / a.ksplit;
  const int group = warp / a.ksplit, kpart = warp - group * a.ksplit;
  const int n0 = (blockIdx.x * groups_per_cta + group) * R;
  const bool active = n0 < a.n;
  const bool norm = a.norm_w != nullptr;
  pdl_trigger();
  float acc[MR][P][R];
#pragma unroll
  for (int m = 0; m < MR; m++)
#pragma unroll
    for (int p = 0; p < P; p++)
#pragma unroll
      for (int r = 0; r < R; r++) acc[m][p][r] = 0.0f;

  const float* wr[P][R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    int col = n0 + r < a.n ? n0 + r : a.n - 1;  // tail columns re-read the last row; their sums are discarded
    if (col < 0) col = 0;
    if (P == 2) {
      wr[0][r] = a.w[0] + (int64_t)col * a.sw[0];
      wr[P - 1][r] = a.w[1] + (int64_t)col * a.sw[1];
    } else {
      int s = 0;
      while (s + 1 < a.nseg && col >= a.seg_start[s + 1]) s++;
      wr[0][r] = a.w[s] + (int64_t)(col - a.seg_start[s]) * a.sw[s];
    }
  }
  const int k_units = VEC ? (a.k >> 2) : a.k;
  const int per = (k_units + a.ksplit - 1) / a.ksplit;
  const int kb = kpart * per, ke = min(k_units, kb + per);
  float4 wv[U][P][R];
  auto load_w = [&](int i) {
#pragma unroll
    for (int u = 0; u < U; u++) {
      int j = i + 32 * u;
#pragma unroll
      for (int p = 0; p < P; p++)
#pragma unroll
        for (int r = 0; r < R; r++)
          wv[u][p][r] = j < ke ? __ldcs(reinterpret_cast<const float4*>(wr[p][r]) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  // the first trip's weights are requested before waiting on the previous kernel (it never writes the weights)
  if (VEC && active) load_w(kb + lane);
  pdl_wait();
  if (norm) {  // the RmsNorm of each x row, shared by the CTA's warps
    for (int m = warp; m < a.rows && m < MR; m += kWarps) {
      float inv = row_inv_rms(a.x + a.xoff[m], a.k, a.eps, VEC);
      if (lane == 0) s_inv[m] = inv;
    }
    __syncthreads();
  }

  if (active && VEC) {
    for (int i = kb + lane; i < ke; i += 32 * U) {
      if (i != kb + lane) load_w(i);
#pragma unroll
      for (int u = 0; u < U; u++) {
        int j = i + 32 * u;
        if (j >= ke) break;
#pragma unroll
        for (int m = 0; m < MR; m++) {
          if (m >= a.rows) break;
          float4 xv = __ldg(reinterpret_cast<const float4*>(a.x + a.xoff[m]) + j);
          if (norm) {  // RmsNorm's (x · inv) · w, each product rounded once
            float inv = s_inv[m];
            float4 nw = __ldg(reinterpret_cast<const float4*>(a.norm_w) + j);
            xv.x = __fmul_rn(__fmul_rn(xv.x, inv), nw.x);
            xv.y = __fmul_rn(__fmul_rn(xv.y, inv), nw.y);
            xv.z = __fmul_rn(__fmul_rn(xv.z, inv), nw.z);
            xv.w = __fmul_rn(__fmul_rn(xv.w, inv), nw.w);
          }
#pragma unroll
          for (int p = 0; p < P; p++)
#pragma unroll
            for (int r = 0; r < R; r++) {
              acc[m][p][r] = fmaf(xv.x, wv[u][p][r].x, acc[m][p][r]);
              acc[m][p][r] = fmaf(xv.y, wv[u][p][r].y, acc[m][p][r]);
              acc[m][p][r] = fmaf(xv.z, wv[u][p][r].z, acc[m][p][r]);
              acc[m][p][r] = fmaf(xv.w, wv[u][p][r].w, acc[m][p][r]);
            }
        }
      }
    }
  } else if (active) {
    for (int i = kb + lane; i < ke; i += 32) {
      float w1[P][R];
#pragma unroll
      for (int p = 0; p < P; p++)
#pragma unroll
        for (int r = 0; r < R; r++) w1[p][r] = __ldcs(wr[p][r] + i);
#pragma unroll
      for (int m = 0; m < MR; m++) {
        if (m >= a.rows) break;
        float xv = __ldg(a.x + a.xoff[m] + i);
        if (norm) xv = __fmul_rn(__fmul_rn(xv, s_inv[m]), __ldg(a.norm_w + i));
#pragma unroll
        for (int p = 0; p < P; p++)
#pragma unroll
          for (int r = 0; r < R; r++) acc[m][p][r] = fmaf(xv, w1[p][r], acc[m][p][r]);
      }
    }
  }

#pragma unroll
  for (int m = 0; m < MR; m++)
#pragma unroll
    for (int p = 0; p < P; p++)
#pragma unroll
      for (int r = 0; r < R; r++) acc[m][p][r] = warp_sum(acc[m][p][r]);

  if (a.ksplit == 1) {
    if (lane == 0 && n0 < a.n) {
#pragma unroll
      for (int m = 0; m < MR; m++) {
        if (m >= a.rows) break;
#pragma unroll
        for (int r = 0; r < R; r++)
          if (n0 + r < a.n) gemv_store(a, m, n0 + r, acc[m][0][r], acc[m][P - 1][r]);
      }
    }
    return;
  }
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MR; m++)
#pragma unroll
      for (int p = 0; p < P; p++)
#pragma unroll
        for (int r = 0; r < R; r++) part[warp][m][p][r] = acc[m][p][r];
  }
  __syncthreads();
  // one thread per (group, m, r): add the K parts in warp order
  for (int t = threadIdx.x; t < groups_per_cta * MR * R; t += kGemvThreads) {
    int g = t / (MR * R), rem = t - g * (MR * R), m = rem / R, r = rem - m * R;
    int col = (blockIdx.x * groups_per_cta + g) * R + r;
    if (m >= a.rows || col >= a.n) continue;
    float s0 = 0.0f, s1 = 0.0f;
    for (int q = 0; q < a.ksplit; q++) {
      s0 += part[g * a.ksplit + q][m][0][r];
      s1 += part[g * a.ksplit + q][m][P - 1][r];
    }
    gemv_store(a, m, col, s0, s1);
  }
}

// ---------------------------------------------------------------- tensor-core path (5..32 rows)
namespace gtc {

using namespace ::pai::tc;

constexpr int kRowsW = 128;      // W rows per tile (UMMA M)
constexpr int kK = 32;           // k per tile: one 128-byte swizzle row of fp32
constexpr int kStages = 4;       // shared-memory ring depth
constexpr int kSlots = 2;        // tensor-memory A slots (hi + lo, 64 columns each)
constexpr int kWBytes = kRowsW * kK * 4;
constexpr int kThreads = 192;    // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 converters / epilogue
constexpr uint32_t kColAcc = 0;

constexpr int kMaxSegs = kGemvMaxSegs;

// The weight segments of one call share a launch: grid x runs over every segment's 128-row tiles in order.
struct Maps {
  CUtensorMap w[kMaxSegs];       // W_s [n_s, k]: 128-row x 32-k boxes, 128-byte swizzle, zero fill
};

struct Args {
  const float* xhi;              // [kt][rows_pad x 32] pre-split, swizzled x tiles
  const float* xlo;
  float* out;                    // row m of split q at out + q * split_stride + m * ldo, segment s from column col_start[s]
  int64_t ldo, split_stride;
  int* error_flag;
  int rows, rows_pad, kt, kt_per_split;
  int tile_start[kMaxSegs + 1];  // first grid-x tile of each segment (unused entries: the tile count)
  int n_seg[kMaxSegs];           // rows of each W segment
  int col_start[kMaxSegs];       // output column of each segment's first row
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <int NP>  // NP: x rows padded to the MMA's N (16 or 32)
__global__ void __launch_bounds__(kThreads) k_gemv_tc(const __grid_constant__ Maps maps, const Args a) {
  constexpr uint32_t kColA = 64;
  constexpr uint32_t kTmemCols = 256;
  constexpr int kXBytes = NP * 128;
  constexpr int kStage = kWBytes + 2 * kXBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStage);
  uint64_t* stage_free = full + kStages;
  uint64_t* conv = stage_free + kStages;
  uint64_t* slot_free = conv + kSlots;
  uint64_t* acc_full = slot_free + kSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this CTA's weight segment (selected with constant indices: a dynamic index into the parameters would copy
  // them to local memory)
  int seg = 0, seg_tile0 = a.tile_start[0], seg_n = a.n_seg[0], seg_col = a.col_start[0];
#pragma unroll
  for (int i = 1; i < kMaxSegs; i++)
    if ((int)blockIdx.x >= a.tile_start[i]) { seg = i; seg_tile0 = a.tile_start[i]; seg_n = a.n_seg[i]; seg_col = a.col_start[i]; }
  const CUtensorMap* wmap = &maps.w[0] + seg;
  const int n0 = ((int)blockIdx.x - seg_tile0) * kRowsW;
  const int split = blockIdx.y;
  const int k0 = split * a.kt_per_split, k1 = min(a.kt, k0 + a.kt_per_split);
  const int nk = k1 - k0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) { mbar_init(&full[s], 1); mbar_init(&stage_free[s], 1); }
    for (int t = 0; t < kSlots; t++) { mbar_init(&conv[t], 4); mbar_init(&slot_free[t], 1); }
    mbar_init(acc_full, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(wmap)) : "memory");
      // the first stages' weight tiles are requested before waiting on the previous kernel (which wrote x's tiles)
      const int pre = nk < kStages ? nk : kStages;
      for (int i = 0; i < pre; i++) {
        mbar_expect_tx(&full[i], kWBytes + 2 * kXBytes);
        tma_load_2d(smem + i * kStage, wmap, (k0 + i) * kK, n0, &full[i]);
      }
      pdl_wait();
      int issued = 0;
      for (int i = 0; i < nk && !s_abort; i++, issued++) {
        int s = i % kStages;
        uint8_t* st = smem + s * kStage;
        if (i >= pre) {
          if (!mbar_wait(&stage_free[s], ((i / kStages) & 1) ^ 1)) { atomicExch(a.error_flag, 41); s_abort = 1; break; }
          mbar_expect_tx(&full[s], kWBytes + 2 * kXBytes);
          tma_load_2d(st, wmap, (k0 + i) * kK, n0, &full[s]);
        }
        size_t xoff = (size_t)(k0 + i) * (kXBytes / 4);
        bulk_g2s(st + kWBytes, a.xhi + xoff, kXBytes, &full[s]);
        bulk_g2s(st + kWBytes + kXBytes, a.xlo + xoff, kXBytes, &full[s]);
      }
      // every copy issued (the pre-issued weight tiles included) must land before the CTA may exit
      if (issued < pre) issued = pre;
      for (int i = (issued > kStages ? issued - kStages : 0); i < issued; i++) mbar_wait(&full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(128, NP);
      for (int i = 0; i < nk && !s_abort; i++) {
        int s = i % kStages, t = i % kSlots;
        if (!mbar_wait(&conv[t], (i / kSlots) & 1) || !mbar_wait(&full[s], (i / kStages) & 1)) {
          atomicExch(a.error_flag, 42); s_abort = 1; break;
        }
        fence_after();
        uint32_t xhi = smem_u32(smem + s * kStage + kWBytes), xlo = xhi + kXBytes;
        uint32_t ahi = tmem + kColA + t * 64, alo = ahi + 32;
#pragma unroll
        for (int kk = 0; kk < kK / 8; kk++) {
          uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          uint32_t d = tmem + kColAcc;
          mma_ts(d, alo + kk * 8, desc_sw128(xhi + kk * 32), idesc, acc);
          mma_ts(d, ahi + kk * 8, desc_sw128(xlo + kk * 32), idesc, 1u);
          mma_ts(d, ahi + kk * 8, desc_sw128(xhi + kk * 32), idesc, 1u);
        }
        commit(&stage_free[s]);
        commit(&slot_free[t]);
      }
      commit(acc_full);
    }
  } else {
    pdl_wait();
    // converters: warp quadrant q owns W rows 32q..32q+31 of the tile (its TMEM lanes)
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    for (int i = 0; i < nk; i++) {
      int s = i % kStages, t = i % kSlots;
      if (!warp_wait(&full[s], (i / kStages) & 1) || !warp_wait(&slot_free[t], ((i / kSlots) & 1) ^ 1)) {
        if (lane == 0) { atomicExch(a.error_flag, 43); s_abort = 1; }
        break;
      }
      fence_after();
      const uint8_t* row = smem + s * kStage + r * 128;
      float hi[32], lo[32];
#pragma unroll
      for (int c = 0; c < 8; c++) {
        float4 v = *reinterpret_cast<const float4*>(row + ((c ^ (r & 7)) << 4));
        split_tf32_fast(v.x, hi[4 * c], lo[4 * c]);
        split_tf32_fast(v.y, hi[4 * c + 1], lo[4 * c + 1]);
        split_tf32_fast(v.z, hi[4 * c + 2], lo[4 * c + 2]);
        split_tf32_fast(v.w, hi[4 * c + 3], lo[4 * c + 3]);
      }
      tmem_st32(tmem + lane_base + kColA + t * 64, hi);
      tmem_st32(tmem + lane_base + kColA + t * 64 + 32, lo);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[t]);
    }
    // epilogue: lane = W row n, TMEM column m = x row
    if (warp_wait(acc_full, 0)) {
      fence_after();
      float v[32];
      tmem_ld32(tmem + lane_base + kColAcc, v);
      const int n = n0 + r;
      float* dst = a.out + (size_t)split * a.split_stride + seg_col;
      if (n < seg_n) {
#pragma unroll
        for (int m = 0; m < NP; m++)
          if (m < a.rows) dst[(size_t)m * a.ldo + n] = v[m];
      }
    } else if (lane == 0) {
      atomicExch(a.error_flag, 44);
      s_abort = 1;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// x rows (element offsets xoff, contiguous along k) -> hi/lo tiles [kt][NP rows x 32 k] in the K-major SWIZZLE_128B
// layout (row r at (r/8)*1024 + (r%8)*128, 16-byte chunk c at chunk c ^ (r%8)); rows >= rows and k >= K are zero.
struct XPack {
  const float* x;
  int64_t xoff[kGemvMaxRows];
  int rows, np, k, kt;
  const float* norm_w;  // when set, each row is RMS-normalised first (RmsNorm's values, bit for bit)
  float eps;
  int vec;              // rows are 16-byte aligned with k a multiple of 4
};

// One CTA per (padded) x row: optional RmsNorm, then the tf32 hi/lo split into the swizzled tiles.
__global__ void __launch_bounds__(256) k_pack_x(const XPack p, float* __restrict__ hi, float* __restrict__ lo) {
  pdl_trigger();
  pdl_wait();
  __shared__ float s_inv;
  const int rr = blockIdx.x;
  const bool real = rr < p.rows;
  const float* src = real ? p.x + p.xoff[rr] : nullptr;
  if (p.norm_w && real) {
    if (threadIdx.x < 32) {
      float inv = row_inv_rms(src, p.k, p.eps, p.vec != 0);
      if (threadIdx.x == 0) s_inv = inv;
    }
    __syncthreads();
  }
  const int chunks = p.kt * 8;  // 16-byte chunks of the row across all k tiles
  for (int i = threadIdx.x; i < chunks; i += blockDim.x) {
    int c = i & 7, kb = i >> 3;
    int k = kb * kK + 4 * c;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (real) {
#pragma unroll
      for (int e = 0; e < 4; e++)
        if (k + e < p.k) {
          float xv = src[k + e];
          if (p.norm_w) xv = __fmul_rn(__fmul_rn(xv, s_inv), p.norm_w[k + e]);
          v[e] = xv;
        }
    }
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; e++) split_tf32(v[e], h[e], l[e]);
    size_t off = (size_t)kb * p.np * 32 + (size_t)(rr >> 3) * 256 + (size_t)(rr & 7) * 32 + (size_t)((c ^ (rr & 7)) * 4);
    *reinterpret_cast<float4*>(hi + off) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + off) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

template <int NP>
constexpr size_t smem_bytes() {
  return (size_t)kStages * (kWBytes + 2 * NP * 128) + 1024 + 256;
}

// Sums the split-K partials (split q of row m at p + q * plane + m * ldp) in split order and applies the epilogue:
// y[m, c] = a (store), res[m, c] + a (residual), SiLU(a)·b (SiLU·mul; b from column colb + c of the same partials).
__global__ void k_gemv_finish(const float* __restrict__ p, int splits, int64_t plane, int64_t ldp, int colb, int rows, int n,
                              float* __restrict__ y, int64_t ldy, int mode, const float* __restrict__ res, int64_t ldr) {
  pdl_trigger();
  pdl_wait();
  const int64_t total = (int64_t)rows * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int m = (int)(i / n), c = (int)(i - (int64_t)m * n);
    const float* pm = p + (int64_t)m * ldp + c;
    float va = pm[0];
    for (int q = 1; q < splits; q++) va += pm[q * plane];
    float out = va;
    if (mode == kGemvResidual) {
      out = __fadd_rn(res[(int64_t)m * ldr + c], va);
    } else if (mode == kGemvSiluMul) {
      float vb = pm[colb];
      for (int q = 1; q < splits; q++) vb += pm[q * plane + colb];
      out = silu_mul_value(va, vb);
    }
    y[(int64_t)m * ldy + c] = out;
  }
}

}  // namespace gtc

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// One weight segment of a fused x·Wᵀ call: W rows [n, k] with row stride sw (unit column stride).
struct LinearSeg {
  const float* w;
  int64_t sw;
  int n;
};

// Tensor-core product of pre-split x tiles against all weight segments in one launch (grid x over the segments'
// 128-row tiles, y over the K splits), then the epilogue: store mode with one split writes y directly (segments side
// by side); otherwise split-K partials [splits][rows, n_total] go to a scratch buffer that k_gemv_finish sums in split
// order with the store / residual / SiLU·mul epilogue.
static pai_status gemv_tc(pai_ctx* ctx, const float* xh, const float* xl, int rows, int np, int k, const LinearSeg* segs,
                          int nseg, int mode, float* y, int64_t ldy, const float* res, int64_t ldr) {
  using namespace gtc;
  auto encode = tensor_map_encoder();
  if (!encode) return set_error(PAI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const int kt = (k + kK - 1) / kK;
  Maps maps;
  memset(&maps, 0, sizeof maps);
  Args a{};
  int tiles = 0, n_total = 0;
  for (int s = 0; s < nseg; s++) {
    const LinearSeg& sg = segs[s];
    // W [n, k] row-major with row stride sw: a 2-D tensor map of 128-row x 32-k boxes, 128-byte swizzle, zero fill
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)sg.n};
    cuuint64_t strides[1] = {(cuuint64_t)sg.sw * 4};
    cuuint32_t box[2] = {(cuuint32_t)kK, (cuuint32_t)kRowsW};
    cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(&maps.w[s], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(sg.w), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS)
      return set_error(PAI_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for W [%d, %d]", (int)cr, sg.n, k);
    a.tile_start[s] = tiles;
    a.n_seg[s] = sg.n;
    a.col_start[s] = n_total;
    n_total += sg.n;
    tiles += (sg.n + kRowsW - 1) / kRowsW;
  }
  for (int s = nseg; s <= kMaxSegs; s++) a.tile_start[s] = tiles;
  int splits = std::max(1, std::min(2 * ctx->sm_count / tiles, kt / 4));
  int ktp = (kt + splits - 1) / splits;
  splits = (kt + ktp - 1) / ktp;
  a.xhi = xh;
  a.xlo = xl;
  a.error_flag = ctx->d_error_flag;
  a.rows = rows;
  a.rows_pad = np;
  a.kt = kt;
  a.kt_per_split = ktp;
  const bool direct = mode == kGemvStore && splits == 1;
  Scratch part;
  if (direct) {
    a.out = y;
    a.ldo = ldy;
  } else {
    PAI_TRY(scratch(ctx, (size_t)splits * rows * n_total * 4, &part));
    a.out = static_cast<float*>(part.p);
    a.ldo = n_total;
    a.split_stride = (int64_t)rows * n_total;
  }
  dim3 grid((unsigned)tiles, (unsigned)splits);
  if (np == 16) {
    PAI_CUDA(smem_limit(ctx, k_gemv_tc<16>, (int)smem_bytes<16>()));
    PAI_PDL_LAUNCH(launch_pdl(k_gemv_tc<16>, grid, dim3(kThreads), smem_bytes<16>(), ctx->stream, maps, a), "gemv tc");
  } else {
    PAI_CUDA(smem_limit(ctx, k_gemv_tc<32>, (int)smem_bytes<32>()));
    PAI_PDL_LAUNCH(launch_pdl(k_gemv_tc<32>, grid, dim3(kThreads), smem_bytes<32>(), ctx->stream, maps, a), "gemv tc");
  }
  if (!direct) {
    const int n_out = mode == kGemvStore ? n_total : segs[0].n;
    const int64_t nn = (int64_t)rows * n_out;
    PAI_PDL_LAUNCH(launch_pdl(k_gemv_finish, dim3(grid_for(ctx, nn, 256)), dim3(256), 0, ctx->stream,
                              static_cast<const float*>(part.p), splits, (int64_t)rows * n_total, (int64_t)n_total,
                              mode == kGemvSiluMul ? segs[0].n : 0, rows, n_out, y, ldy, mode, res, ldr),
                   "gemv finish");
  }
  return PAI_OK;
}

template <int MR, int U, int P>
static pai_status launch_gemv_mr(pai_ctx* ctx, const GemvArgs& g, bool vec, int grid) {
  cudaError_t e = vec ? launch_pdl(k_gemv_tn<MR, U, true, P>, dim3(grid), dim3(kGemvThreads), 0, ctx->stream, g)
                      : launch_pdl(k_gemv_tn<MR, U, false, P>, dim3(grid), dim3(kGemvThreads), 0, ctx->stream, g);
  if (e != cudaSuccess) return cuda_error(e, "gemv");
  ctx->launches++;
  return PAI_OK;
}

template <int P>
static pai_status launch_gemv(pai_ctx* ctx, const GemvArgs& g, bool vec, int grid) {
  constexpr int U1 = P == 1 ? 4 : 2;
  if (g.rows == 1) return launch_gemv_mr<1, U1, P>(ctx, g, vec, grid);
  if (g.rows == 2) return launch_gemv_mr<2, U1, P>(ctx, g, vec, grid);
  if (g.rows <= 4) return launch_gemv_mr<4, (P == 1 ? 4 : 1), P>(ctx, g, vec, grid);
  if (g.rows <= 8) return launch_gemv_mr<8, (P == 1 ? 2 : 1), P>(ctx, g, vec, grid);
  if (g.rows <= 16) return launch_gemv_mr<16, 1, P>(ctx, g, vec, grid);
  if (P == 1) return launch_gemv_mr<32, 1, 1>(ctx, g, vec, grid);
  return set_error(PAI_ERR_ARGUMENT, "paired gemv takes at most 16 rows per launch");
}

// rows (<= 32) of x (element offsets xoff, each contiguous along k) against the weight segments, with an epilogue:
//   store:    y[:, seg_start(s) + j] = x · W_sᵀ   (segments side by side)
//   residual: y = res + x · W_0ᵀ
//   SiLU·mul: y = SiLU(x · W_0ᵀ) · (x · W_1ᵀ)   (W_0, W_1 of one shape)
// Output row m at y + m * ldy; residual row m at res + m * ldr.
pai_status linear_rows(pai_ctx* ctx, const float* x, const int64_t* xoff, int rows, int k, const LinearSeg* segs, int nseg,
                       int mode, float* y, int64_t ldy, const float* res, int64_t ldr, const float* norm_w, float eps) {
  if (rows < 1 || rows > kGemvMaxRows) return set_error(PAI_ERR_ARGUMENT, "gemv supports 1..%d rows", kGemvMaxRows);
  if (nseg < 1 || nseg > kGemvMaxSegs) return set_error(PAI_ERR_ARGUMENT, "gemv supports 1..%d weight segments", kGemvMaxSegs);
  if (mode == kGemvSiluMul && (nseg != 2 || segs[0].n != segs[1].n))
    return set_error(PAI_ERR_ARGUMENT, "SiLU·mul needs two weights of one shape");
  if (mode == kGemvResidual && nseg != 1) return set_error(PAI_ERR_ARGUMENT, "the residual epilogue takes one weight");
  bool vec = (k % 4 == 0) && ((uintptr_t)x % 16 == 0);
  int n_total = 0;
  double wbytes = 0;
  for (int s = 0; s < nseg; s++) {
    if (segs[s].sw % 4 || (uintptr_t)segs[s].w % 16) vec = false;
    n_total += segs[s].n;
    wbytes += 4.0 * segs[s].n * (double)k;
  }
  for (int i = 0; i < rows; i++)
    if (xoff[i] % 4) vec = false;
  if (norm_w && (uintptr_t)norm_w % 16) vec = false;
  const int n_out = mode == kGemvStore ? n_total : segs[0].n;
  KernelTimerScope timer(ctx, "gemv", wbytes + 4.0 * rows * (k + n_out));
  if (vec && rows >= kGemvTcMinRows) {
    // tensor cores: split x once, one launch over every weight segment, then the epilogue with the split-K sum
    using namespace gtc;
    const int np = rows <= 16 ? 16 : 32;
    const int kt = (k + kK - 1) / kK;
    Scratch xh, xl;
    size_t xbytes = (size_t)kt * np * kK * 4;
    PAI_TRY(scratch(ctx, xbytes, &xh));
    PAI_TRY(scratch(ctx, xbytes, &xl));
    XPack xp{};
    xp.x = x; xp.rows = rows; xp.np = np; xp.k = k; xp.kt = kt;
    xp.norm_w = norm_w; xp.eps = eps; xp.vec = vec ? 1 : 0;
    for (int i = 0; i < rows; i++) xp.xoff[i] = xoff[i];
    PAI_PDL_LAUNCH(launch_pdl(k_pack_x, dim3(np), dim3(256), 0, ctx->stream, xp, static_cast<float*>(xh.p),
                              static_cast<float*>(xl.p)), "gemv x pack");
    return gemv_tc(ctx, static_cast<const float*>(xh.p), static_cast<const float*>(xl.p), rows, np, k, segs, nseg, mode, y,
                   ldy, res, ldr);
  }

  if (mode == kGemvSiluMul && rows > 16) {
    // the paired kernel holds 16 rows of accumulators: two launches of up to 16 rows each
    PAI_TRY(linear_rows(ctx, x, xoff, 16, k, segs, nseg, mode, y, ldy, res, ldr, norm_w, eps));
    return linear_rows(ctx, x, xoff + 16, rows - 16, k, segs, nseg, mode, y + 16 * ldy, ldy, res ? res + 16 * ldr : nullptr,
                       ldr, norm_w, eps);
  }
  GemvArgs g{};
  g.nseg = nseg;
  int start = 0;
  for (int s = 0; s < nseg; s++) {
    g.w[s] = segs[s].w;
    g.sw[s] = segs[s].sw;
    g.seg_start[s] = start;
    start += segs[s].n;
  }
  g.seg_start[nseg] = start;
  g.x = x; g.y = y; g.ldy = ldy; g.res = res; g.ldr = ldr;
  g.rows = rows; g.n = n_out; g.k = k; g.mode = mode;
  g.norm_w = norm_w; g.eps = eps;
  for (int i = 0; i < rows; i++) g.xoff[i] = xoff[i];
  const int groups = (n_out + kGemvRowsPerWarp - 1) / kGemvRowsPerWarp;
  const int k_units = vec ? k / 4 : k;
  int ksplit = 1;
  // more warps per row group while the grid still fits one resident wave (two 8-warp CTAs per SM) and each lane keeps
  // >= 2 loads per row: every warp then issues its loads at once and no CTA waits for a second wave
  while (ksplit < 8 && (int64_t)groups * ksplit * 2 <= (int64_t)ctx->sm_count * 16 && k_units / (ksplit * 2) >= 64) ksplit *= 2;
  g.ksplit = ksplit;
  const int groups_per_cta = (kGemvThreads / 32) / ksplit;
  const int grid = (groups + groups_per_cta - 1) / groups_per_cta;
  return mode == kGemvSiluMul ? launch_gemv<2>(ctx, g, vec, grid) : launch_gemv<1>(ctx, g, vec, grid);
}

// y (dense [rows, n]) = rows of x · Wᵀ (the MatMul path for decode-sized products).
pai_status gemv_tn(pai_ctx* ctx, const float* x, const int64_t* xoff, int rows, const float* w, int64_t sw, int n, int k,
                   float* y) {
  LinearSeg sg{w, sw, n};
  return linear_rows(ctx, x, xoff, rows, k, &sg, 1, kGemvStore, y, n, nullptr, 0, nullptr, 0.0f);
}

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_linear_fused(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* norm_weight, float eps,
                                    const pai_tensor* weights, int32_t n_weights, int32_t mode, const pai_tensor* residual,
                                    pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  if (x->rank < 1 || x->strides[x->rank - 1] != 1)
    return set_error(PAI_ERR_ARGUMENT, "LinearFused: x must have rank >= 1 and contiguous rows");
  if (n_weights < 1 || n_weights > kGemvMaxSegs || !weights)
    return set_error(PAI_ERR_ARGUMENT, "LinearFused: 1..%d weights expected", kGemvMaxSegs);
  if (mode < kGemvStore || mode > kGemvSiluMul) return set_error(PAI_ERR_ARGUMENT, "LinearFused: unknown mode %d", mode);
  const int k = x->dims[x->rank - 1];
  const int64_t rows64 = k ? numel(*x) / k : 0;
  if (rows64 < 1 || rows64 > kGemvMaxRows)
    return set_error(PAI_ERR_ARGUMENT, "LinearFused: %lld rows; 1..%d supported", (long long)rows64, kGemvMaxRows);
  const int rows = (int)rows64;
  LinearSeg segs[kGemvMaxSegs];
  int n_total = 0;
  for (int i = 0; i < n_weights; i++) {
    const pai_tensor& w = weights[i];
    PAI_TRY(check_view(ctx, &w, "weight"));
    if (w.rank != 2 || w.dims[1] != k || w.strides[1] != 1)
      return set_error(PAI_ERR_ARGUMENT, "LinearFused: weight %d must be [n, %d] with contiguous rows, got %s", i, k,
                       shape_str(w).c_str());
    segs[i] = LinearSeg{fptr(w), w.strides[0], w.dims[0]};
    n_total += w.dims[0];
  }
  const int n_out = mode == kGemvStore ? n_total : segs[0].n;
  const float* res = nullptr;
  int64_t ldr = 0;
  if (mode == kGemvResidual) {
    if (!residual) return set_error(PAI_ERR_ARGUMENT, "LinearFused: the residual mode needs a residual tensor");
    PAI_TRY(check_view(ctx, residual, "residual"));
    if (!is_dense(*residual) || numel(*residual) != (int64_t)rows * n_out)
      return set_error(PAI_ERR_ARGUMENT, "LinearFused: residual must be a dense [%d, %d]", rows, n_out);
    res = fptr(*residual);
    ldr = n_out;
  }
  // per-row element offsets of x over its leading dims
  int64_t xoff[kGemvMaxRows];
  for (int r = 0; r < rows; r++) {
    int64_t rem = r, off = x->offset;
    for (int d = x->rank - 2; d >= 0; d--) {
      off += (rem % x->dims[d]) * x->strides[d];
      rem /= x->dims[d];
    }
    xoff[r] = off;
  }
  const float* nw = nullptr;
  if (norm_weight) {
    PAI_TRY(check_view(ctx, norm_weight, "norm weight"));
    if (norm_weight->rank != 1 || norm_weight->dims[0] != k || norm_weight->strides[0] != 1)
      return set_error(PAI_ERR_ARGUMENT, "LinearFused: the norm weight must be a contiguous [%d]", k);
    nw = fptr(*norm_weight);
  }
  int32_t od[PAI_MAX_RANK];
  for (int i = 0; i < x->rank - 1; i++) od[i] = x->dims[i];
  od[x->rank - 1] = n_out;
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, x->rank, od, x->dtype, false, &r));
  PAI_TRY(linear_rows(ctx, static_cast<const float*>(x->base), xoff, rows, k, segs, n_weights, mode, fptr(r), n_out, res, ldr,
                      nw, eps));
  *out = r;
  return PAI_OK;
}
