// Batched GEMM for IComputeBackend.MatMul (IComputeBackend.cs:33-35; semantics CpuComputeBackend.cs:159-219):
// C[b] = A[b] · B[b] (or · B[b]ᵀ), NumPy batch broadcasting, arbitrary operand views.
//
// fp32 semantics on the tensor cores (3xTF32): every operand element x is split into hi = tf32(x) and
// lo = tf32(x − hi) (round-to-nearest, both exactly representable in tf32), and each product is accumulated as
// a_lo·b_hi + a_hi·b_lo + a_hi·b_hi in an fp32 TMEM accumulator. The dropped a_lo·b_lo term and the tf32 rounding
// of lo leave a relative error near 2^-21 per product, well inside the 1e-4 conformance tolerance. The tensor core
// reads an fp32 operand as tf32 by dropping its low 13 mantissa bits, so for a K-major operand of the two-CTA kernel
// hi is the operand itself and lo = tf32(x − trunc(x)): one plane is written instead of two (the dropped lo·lo term
// is then below 2^-20 relative).
//
// Pipeline:
//   1. k_pack: both operands in one launch (the smaller one's tiles first); reads each operand view once (any
//      strides, batch offsets), splits hi/lo, and writes 128-row x 32-k
//      tiles already in the tcgen05 K-major SWIZZLE_128B shared-memory layout, so the GEMM moves each tile with
//      one plain bulk copy (cp.async.bulk) and no tensor map. A K-major operand of the two-CTA kernel gets its lo
//      plane only; its hi tiles come from the operand through a SWIZZLE_128B tensor map.
//   2. k_gemm_tc: persistent kernel, one CTA per SM, warp-specialised:
//        warp 0   bulk-copy producer into a STAGES-deep shared-memory ring (mbarrier complete_tx);
//        warp 1   allocates TMEM and issues tcgen05.mma.kind::tf32 (M=128, N=BN) from one elected lane;
//        warps 2-5 epilogue: tcgen05.ld from a double-buffered TMEM accumulator, fp32 stores to C.
//      Split-K (partials + deterministic reduce) keeps the SMs busy on deep-K, small-MN products (weight grads).
//   Every mbarrier wait is bounded; a timeout sets the context's device error flag and the kernel drains and exits.
#include <stdlib.h>
#include <string.h>

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "common.cuh"

namespace pai {

constexpr int kBM = 128;                        // UMMA M (rows of A per tile)
constexpr int kBK = 32;                         // fp32 elements per 128-byte swizzle row
constexpr int kTileFloats = kBM * kBK;          // one packed 128x32 tile (16 KiB)
constexpr uint32_t kWaitLimit = 1u << 26;       // bounded mbarrier polls before declaring a hang

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Returns false if the phase did not complete within the poll budget.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kWaitLimit; i++) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// tcgen05 shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);           // start address
  d |= (uint64_t)1 << 16;                            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::tf32, fp32 accumulate, A and B K-major, M = bm (128, or 256 for a CTA pair), N = bn.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int bn, int bm = kBM) {
  return (1u << 4)                    // D format: f32
         | (2u << 7)                  // A format: tf32
         | (2u << 10)                 // B format: tf32
         | ((uint32_t)(bn >> 3) << 17)  // N >> 3
         | ((uint32_t)(bm >> 4) << 24);  // M >> 4
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive TMEM columns of this warp's 32 lanes -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- pack
// Up to this many batch matrices travel inside the kernel parameters (read through a __grid_constant__ parameter, so
// in place); more take a device array uploaded per call. Inline arrays keep the host-to-device copies (each one a
// copy-engine operation serialised between kernels on the stream) off the per-product path.
constexpr int kInlineBatches = 16;

struct PackDesc {
  const float* src;
  const int64_t* batch_off;  // element offset of each batch matrix (device array), or null: boff_inline holds them
  int64_t boff_inline[kInlineBatches];
  int64_t sr, sk;            // element strides along rows and along k
  int rows, k;               // logical extent
  int kt, rt_pad;            // k tiles, row tiles (padded)
  int vec;                   // 1: 16-byte loads along the unit-stride axis are aligned and never straddle an edge
  int lo_only;               // 1: the GEMM reads the raw fp32 operand as hi (the tensor core truncates it to tf32),
                             //    so only lo = tf32(x − trunc(x)) is written
};

// One CTA (256 threads) writes one 128x32 hi tile and one lo tile: k tile kt, row tile rt, batch matrix b.
__device__ __forceinline__ void pack_tile(const PackDesc& d, int kt, int rt, int b, float* __restrict__ hi,
                                          float* __restrict__ lo) {
  __shared__ float tile[kBM][kBK + 1];
  int tid = threadIdx.x;
  const int64_t* boffs = d.batch_off ? d.batch_off : d.boff_inline;
  const float* src = d.src + boffs[b];
  int r0 = rt * kBM, k0 = kt * kBK;
  if (d.vec && d.sk == 1) {
    for (int idx = tid; idx < kBM * (kBK / 4); idx += 256) {
      int r = idx >> 3, k = (idx & 7) * 4;
      int gr = r0 + r, gk = k0 + k;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gr < d.rows && gk < d.k) v = *reinterpret_cast<const float4*>(src + (int64_t)gr * d.sr + gk);
      tile[r][k] = v.x; tile[r][k + 1] = v.y; tile[r][k + 2] = v.z; tile[r][k + 3] = v.w;
    }
  } else if (d.vec && d.sr == 1) {
    for (int idx = tid; idx < (kBM / 4) * kBK; idx += 256) {
      int r = (idx & 31) * 4, k = idx >> 5;
      int gr = r0 + r, gk = k0 + k;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gr < d.rows && gk < d.k) v = *reinterpret_cast<const float4*>(src + gr + (int64_t)gk * d.sk);
      tile[r][k] = v.x; tile[r + 1][k] = v.y; tile[r + 2][k] = v.z; tile[r + 3][k] = v.w;
    }
  } else if (d.sk == 1) {
    for (int idx = tid; idx < kBM * kBK; idx += 256) {
      int r = idx >> 5, k = idx & 31;
      int gr = r0 + r, gk = k0 + k;
      tile[r][k] = (gr < d.rows && gk < d.k) ? src[(int64_t)gr * d.sr + gk] : 0.0f;
    }
  } else {
    for (int idx = tid; idx < kBM * kBK; idx += 256) {
      int r = idx & (kBM - 1), k = idx >> 7;
      int gr = r0 + r, gk = k0 + k;
      tile[r][k] = (gr < d.rows && gk < d.k) ? src[(int64_t)gr * d.sr + (int64_t)gk * d.sk] : 0.0f;
    }
  }
  __syncthreads();
  size_t base = ((size_t)(b * d.kt + kt) * d.rt_pad + rt) * kTileFloats;
  float4* l4 = reinterpret_cast<float4*>(lo + base);
  if (d.lo_only) {
    // hi is the raw value as the tensor core reads it (low 13 mantissa bits dropped); x − hi is exact.
    for (int ch = tid; ch < kBM * 8; ch += 256) {
      int r = ch >> 3, c = ch & 7;
      float vl[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float v = tile[r][c * 4 + j];
        vl[j] = __uint_as_float(to_tf32(v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u)));
      }
      l4[r * 8 + (c ^ (r & 7))] = make_float4(vl[0], vl[1], vl[2], vl[3]);
    }
    return;
  }
  float4* h4 = reinterpret_cast<float4*>(hi + base);
  for (int ch = tid; ch < kBM * 8; ch += 256) {
    int r = ch >> 3, c = ch & 7;
    float v[4], vh[4], vl[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      v[j] = tile[r][c * 4 + j];
      uint32_t h = to_tf32(v[j]);
      vh[j] = __uint_as_float(h);
      vl[j] = __uint_as_float(to_tf32(v[j] - vh[j]));
    }
    int phys = r * 8 + (c ^ (r & 7));  // SWIZZLE_128B: 16-byte chunk index XOR row within the 8-row group
    h4[phys] = make_float4(vh[0], vh[1], vh[2], vh[3]);
    l4[phys] = make_float4(vl[0], vl[1], vl[2], vl[3]);
  }
}

// Both operands of a product in one launch: CTAs [0, tiles0) pack operand 0, the rest operand 1, each walking its
// (k tile, row tile, batch) space k tile fastest. The weight operand goes first, so its small pack overlaps the
// activation's instead of paying a launch of its own.
struct PackPair {
  PackDesc d[2];
  float* hi[2];
  float* lo[2];
  int64_t tiles0;
};

__global__ void __launch_bounds__(256) k_pack(const __grid_constant__ PackPair p) {
  int64_t i = blockIdx.x;
  const int o = i < p.tiles0 ? 0 : 1;
  if (o) i -= p.tiles0;
  const PackDesc& d = p.d[o];
  const int kt = (int)(i % d.kt);
  const int64_t rest = i / d.kt;
  const int rt = (int)(rest % d.rt_pad);
  const int b = (int)(rest / d.rt_pad);
  pack_tile(d, kt, rt, b, p.hi[o], p.lo[o]);
}

// ---------------------------------------------------------------- tcgen05 GEMM
struct GemmArgs {
  const float* a_hi; const float* a_lo;  // packed A: [batch_a][kt][mt_pad][tile]
  const float* b_hi; const float* b_lo;  // packed B: [batch_b][kt][nt_pad][tile]
  const int32_t* a_index;                // output batch -> A batch (device array), or null: the inline arrays
  const int32_t* b_index;                // output batch -> B batch
  int32_t a_index_inline[kInlineBatches];
  int32_t b_index_inline[kInlineBatches];
  float* c;                              // [batch][m][n] (or split partials [split][batch][m][n])
  int m, n, kt;                          // rows, cols, k tiles
  int mt_pad, nt_pad;                    // 128-row tiles of the packed A and B
  int tiles_m, tiles_n, batches, splits; // output tiles (kTileM x kTileN) per batch, K splits
  int kt_per_split;
  int* error_flag;
  int k_elems;                           // logical K (for the work count only)
  int a_raw, b_raw;                      // pair kernel: hi is read from the raw operand (its tensor map), not a plane
};

// The CTA-pair kernel reads the same packed planes through 2-D tensor maps ([rows, 32] fp32, 128-row boxes, no
// swizzle: each box is one pre-swizzled tile copied verbatim), so the partner CTA's copies can signal the leader's
// barrier (the .cta_group::2 form of the tensor copy). A K-major operand's hi map may instead cover the raw operand
// ([rows, k] fp32, 32 x 128 boxes, SWIZZLE_128B): the copy then lays the tile out as the pack would, and rows or k
// past the edge read as zeros, as the pack pads them.
struct PairMaps {
  CUtensorMap a_hi, a_lo, b_hi, b_lo;
};

constexpr int kTileN = 256;        // output columns per tile (one MMA's N)
constexpr int kEpiWarps = 8;       // two per TMEM lane quadrant, each owning half of a row's 256 columns
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kPartialCols = 256;  // one TMEM partial accumulator (128 lanes x 256 fp32 columns); two stages
constexpr int kPromoteKt = 8;           // k tiles (32 wide) summed in TMEM before the epilogue folds the partial into fp32

template <bool PAIR>
struct GemmShape {
  static constexpr int kTileM = PAIR ? 256 : 128;   // output rows per tile (a CTA pair computes 256 x 256)
  static constexpr int kBRows = PAIR ? 128 : 256;   // B rows (output columns) each CTA stages per k tile
  static constexpr int kA = kBM * kBK * 4;          // 16 KiB
  static constexpr int kB = kBRows * kBK * 4;       // 16 or 32 KiB
  static constexpr int kStage = 2 * kA + 2 * kB;    // hi and lo planes of both operands
  static constexpr int kStages = PAIR ? 3 : 2;
  static constexpr int kBytes = kStages * kStage + 1024 /*align*/ + 256 /*barriers*/;
};

// Tile order: split-K slice, then batch, then a grouped raster over (m, n) — kGroupM row tiles walked first inside
// each column band — so the tiles in flight at once share a few A row-blocks and B column-blocks in L2 instead of each
// streaming its own operands from HBM.
constexpr int kGroupM = 16;

__device__ __forceinline__ void tile_coords(const GemmArgs& g, int t, int& split, int& bt, int& mb, int& nb) {
  int per_split = g.tiles_m * g.tiles_n * g.batches;
  split = t / per_split;
  int rem = t % per_split;
  bt = rem / (g.tiles_m * g.tiles_n);
  int r2 = rem % (g.tiles_m * g.tiles_n);
  int span = kGroupM * g.tiles_n;
  int group = r2 / span;
  int first_m = group * kGroupM;
  int gsize = min(g.tiles_m - first_m, kGroupM);
  int within = r2 % span;
  mb = first_m + within % gsize;
  nb = within / gsize;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// mbar_wait with cluster-scope acquire: the barrier also receives arrivals from the partner CTA.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kWaitLimit; i++) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
// Lane 0 polls, the warp follows (keeps the .sync.aligned TMEM loads convergent on every path).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
// One 128-row box (at element x of the row, a multiple of 32) into this CTA's shared memory; the bytes count on the
// leader CTA's barrier.
__device__ __forceinline__ void tma_pair_load(void* dst, const CUtensorMap* map, int x, int row, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(row), "r"(bar_cluster)
      : "memory");
}
template <bool PAIR>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  if (PAIR)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
  else
    umma_tf32(d_tmem, a, b, idesc, accumulate);
}
// Completion of the MMAs issued so far arrives on `bar` (PAIR: on the barrier at that offset in both CTAs).
template <bool PAIR>
__device__ __forceinline__ void umma_commit_all(uint64_t* bar) {
  if (PAIR)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(smem_u32(bar)), "h"((uint16_t)3) : "memory");
  else
    umma_commit(bar);
}

// Persistent, warp-specialised 3xTF32 GEMM. PAIR = false: one CTA per SM, 128 x 256 output tiles. PAIR = true: a
// cluster of two CTAs (one per SM) computes 256 x 256 tiles with cta_group::2 MMAs (M = 256: each CTA holds 128 rows
// of A and of the accumulator, and stages half of B's 256 columns, so each SM reads half of B per MMA).
//   warp 0      copies A and B tiles (hi and lo planes) into a ring of shared-memory stages;
//   warp 1      allocates TMEM and (the leader CTA's lane 0) issues the MMAs;
//   warps 2-9   accumulate and store the result.
// Accuracy: the tensor core sums into its fp32 accumulator with a rounding that does not average out over thousands of
// accumulations (at K = 5632 a single accumulator lands ~30x further from the float64 result than a sequential fp32
// loop). So every kPromoteKt k tiles go into a fresh TMEM partial (two stages, ping-pong), with the small cross terms
// (a_lo·b_hi, a_hi·b_lo) issued before the large a_hi·b_hi, and the epilogue warps add each partial into fp32
// registers with IEEE round-to-nearest: per-partial errors have random signs and average out across the partials.
template <bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm_tc(const __grid_constant__ GemmArgs g,
                                                             const __grid_constant__ PairMaps maps) {
  using S = GemmShape<PAIR>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStage);
  uint64_t* empty_bar = full_bar + S::kStages;
  uint64_t* part_full = empty_bar + S::kStages;
  uint64_t* part_empty = part_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(part_empty + 2);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; s++) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
    for (int a = 0; a < 2; a++) { mbar_init(&part_full[a], 1); mbar_init(&part_empty[a], PAIR ? 2 * kEpiWarps : kEpiWarps); }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(2 * kPartialCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(2 * kPartialCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // both CTAs' barriers exist before any copy or commit targets them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int total = g.tiles_m * g.tiles_n * g.batches * g.splits;
  const int tiles_per_split = g.tiles_m * g.tiles_n * g.batches;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t lead_full = PAIR ? mapa_rank(smem_u32(&full_bar[0]), 0) : 0u;
      for (int t = unit; t < total && !s_abort; t += units) {
        int split, bt, mb, nb;
        tile_coords(g, t, split, bt, mb, nb);
        const int ba = (g.a_index ? g.a_index : g.a_index_inline)[bt];
        const int bb = (g.b_index ? g.b_index : g.b_index_inline)[bt];
        const int k0 = split * g.kt_per_split, k1 = min(g.kt, k0 + g.kt_per_split);
        for (int kb = k0; kb < k1; kb++) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { atomicExch(g.error_flag, 1); s_abort = 1; break; }
          uint8_t* st = smem + stage * S::kStage;
          if (PAIR) {
            if (leader) mbar_expect_tx(&full_bar[stage], 2u * (uint32_t)S::kStage);
            const uint32_t bar = lead_full + (uint32_t)(stage * 8);
            const int arow = ((ba * g.kt + kb) * g.mt_pad + mb * 2 + (int)rank) * kBM;
            const int brow = ((bb * g.kt + kb) * g.nt_pad + nb * 2 + (int)rank) * kBM;
            if (g.a_raw) tma_pair_load(st, &maps.a_hi, kb * kBK, (mb * 2 + (int)rank) * kBM, bar);
            else tma_pair_load(st, &maps.a_hi, 0, arow, bar);
            tma_pair_load(st + S::kA, &maps.a_lo, 0, arow, bar);
            if (g.b_raw) tma_pair_load(st + 2 * S::kA, &maps.b_hi, kb * kBK, (nb * 2 + (int)rank) * kBM, bar);
            else tma_pair_load(st + 2 * S::kA, &maps.b_hi, 0, brow, bar);
            tma_pair_load(st + 2 * S::kA + S::kB, &maps.b_lo, 0, brow, bar);
          } else {
            mbar_expect_tx(&full_bar[stage], (uint32_t)S::kStage);
            const size_t aoff = ((size_t)(ba * g.kt + kb) * g.mt_pad + mb) * kTileFloats;
            const size_t boff = ((size_t)(bb * g.kt + kb) * g.nt_pad + (size_t)nb * 2) * kTileFloats;
            bulk_g2s(st, g.a_hi + aoff, S::kA, &full_bar[stage]);
            bulk_g2s(st + S::kA, g.a_lo + aoff, S::kA, &full_bar[stage]);
            bulk_g2s(st + 2 * S::kA, g.b_hi + boff, S::kB, &full_bar[stage]);
            bulk_g2s(st + 2 * S::kA + S::kB, g.b_lo + boff, S::kB, &full_bar[stage]);
          }
          if (++stage == S::kStages) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: every stage issued must have landed (and been consumed) before the CTA may exit.
      for (int s = 0; s < S::kStages; s++) {
        mbar_wait(&empty_bar[stage], phase ^ 1);
        if (++stage == S::kStages) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_tf32(kTileN, S::kTileM);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t J = 0;  // running partial count: partial stage J & 1, its barrier phase (J >> 1) & 1
      for (int t = unit; t < total && !s_abort; t += units) {
        const int split = t / tiles_per_split;
        const int k0 = split * g.kt_per_split, k1 = min(g.kt, k0 + g.kt_per_split);
        for (int kb = k0; kb < k1; kb++) {
          const int ps = (int)(J & 1);
          const bool first = (kb - k0) % kPromoteKt == 0;
          const bool last = (kb - k0) % kPromoteKt == kPromoteKt - 1 || kb == k1 - 1;
          if (!mbar_wait(&full_bar[stage], phase)) { atomicExch(g.error_flag, 3); s_abort = 1; break; }
          if (first) {
            const bool freed = PAIR ? mbar_wait_cluster(&part_empty[ps], ((J >> 1) & 1) ^ 1)
                                    : mbar_wait(&part_empty[ps], ((J >> 1) & 1) ^ 1);
            if (!freed) { atomicExch(g.error_flag, 2); s_abort = 1; break; }
          }
          tc_fence_after();
          uint8_t* st = smem + stage * S::kStage;
          const uint32_t a_hi = smem_u32(st), a_lo = a_hi + S::kA, b_hi = a_hi + 2 * S::kA, b_lo = b_hi + S::kB;
          const uint32_t d = tmem_base + (uint32_t)ps * kPartialCols;
#pragma unroll
          for (int ks = 0; ks < kBK / 8; ks++) {
            const uint32_t ko = (uint32_t)ks * 32;  // 8 tf32 = 32 bytes along K inside the 128-byte swizzle row
            umma<PAIR>(d, umma_desc_sw128(a_lo + ko), umma_desc_sw128(b_hi + ko), idesc, (first && ks == 0) ? 0u : 1u);
            umma<PAIR>(d, umma_desc_sw128(a_hi + ko), umma_desc_sw128(b_lo + ko), idesc, 1u);
          }
#pragma unroll
          for (int ks = 0; ks < kBK / 8; ks++) {
            const uint32_t ko = (uint32_t)ks * 32;
            umma<PAIR>(d, umma_desc_sw128(a_hi + ko), umma_desc_sw128(b_hi + ko), idesc, 1u);
          }
          umma_commit_all<PAIR>(&empty_bar[stage]);  // frees the stage (in both CTAs) once these MMAs have read it
          if (last) {
            umma_commit_all<PAIR>(&part_full[ps]);
            J++;
          }
          if (++stage == S::kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else {
    // Epilogue warps 2..9: TMEM lane quadrant = warp % 4, column half = (warp - 2) / 4 (128 of the tile's 256).
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * (kTileN / 2));
    const uint32_t lead_part_empty = PAIR ? mapa_rank(smem_u32(&part_empty[0]), 0) : 0u;
    bool ok = true;
    uint32_t J = 0;
    for (int t = unit; t < total && ok; t += units) {
      int split, bt, mb, nb;
      tile_coords(g, t, split, bt, mb, nb);
      const int k0 = split * g.kt_per_split, k1 = min(g.kt, k0 + g.kt_per_split);
      float acc[kTileN / 2];
#pragma unroll
      for (int j = 0; j < kTileN / 2; j++) acc[j] = 0.0f;
      const int parts = (k1 - k0 + kPromoteKt - 1) / kPromoteKt;
      for (int pi = 0; pi < parts; pi++, J++) {
        const int ps = (int)(J & 1);
        if (!warp_wait(&part_full[ps], (J >> 1) & 1)) {
          if (lane == 0) { atomicExch(g.error_flag, 4); s_abort = 1; }
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < kTileN / 2 / 16; cc++) {
          float v[16];
          tmem_ld16(lane_base + (uint32_t)ps * kPartialCols + (uint32_t)(cc * 16), v);
#pragma unroll
          for (int j = 0; j < 16; j++) acc[cc * 16 + j] += v[j];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR && !leader) mbar_arrive_remote(lead_part_empty + (uint32_t)(ps * 8));
          else mbar_arrive(&part_empty[ps]);
        }
      }
      if (!ok) break;
      const int row = mb * S::kTileM + (int)rank * kBM + quad * 32 + lane;
      const int col0 = nb * kTileN + half * (kTileN / 2);
      if (row < g.m) {
        float* crow = g.c + ((size_t)split * g.batches + bt) * (size_t)g.m * g.n + (size_t)row * g.n;
        if ((g.n & 3) == 0 && col0 + kTileN / 2 <= g.n) {
          float4* dst = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
          for (int j = 0; j < kTileN / 8; j++) dst[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < kTileN / 2; j++)
            if (col0 + j < g.n) crow[col0 + j] = acc[j];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the partner's MMAs and reads of this CTA's TMEM and shared memory are over
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * kPartialCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * kPartialCols));
  }
}

// Deterministic split-K reduction: c[i] = Σ_s part[s][i] in split order.
__global__ void k_splitk_reduce(const float* __restrict__ part, float* __restrict__ c, int64_t n, int splits) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = part[i];
    for (int s = 1; s < splits; s++) acc += part[(int64_t)s * n + i];
    c[i] = acc;
  }
}

// ---------------------------------------------------------------- host side
pai_status gemv_tn(pai_ctx* ctx, const float* x, const int64_t* xoff, int rows, const float* w, int64_t sw, int n, int k,
                   float* y);

// gemv.cu: the driver's cuTensorMapEncodeTiled, or null.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// A packed plane ([tiles x 128 rows] x 32 fp32, 128-byte rows) as a 2-D tensor map with one-tile boxes.
static pai_status plane_map(const float* plane, int64_t rows, CUtensorMap* map) {
  auto encode = tensor_map_encoder();
  if (!encode) return set_error(PAI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)kBK, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kBK * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  cuuint32_t estr[2] = {1, 1};
  CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(plane), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return set_error(PAI_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for a packed plane", (int)cr);
  return PAI_OK;
}

// A K-major operand in place ([rows, k] fp32, row stride sr elements) as a 2-D tensor map with 32 x 128 boxes in the
// SWIZZLE_128B layout of a packed tile; rows and k past the edge read as zeros.
static pai_status raw_map(const float* base, int rows, int k, int64_t sr, CUtensorMap* map) {
  auto encode = tensor_map_encoder();
  if (!encode) return set_error(PAI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)sr * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  cuuint32_t estr[2] = {1, 1};
  CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return set_error(PAI_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for an operand", (int)cr);
  return PAI_OK;
}

// Whether the pair kernel can read an operand's hi straight from the operand: one matrix, unit stride along k, and
// the base and every row start 16-byte aligned (the tensor map's rules; k a multiple of 4 keeps the row stride legal
// for any row count).
static bool raw_operand_ok(const float* base, const std::vector<int64_t>& distinct, int64_t sr, int64_t sk, int k) {
  if (distinct.size() != 1 || sk != 1 || k % 4 != 0 || sr < k || sr % 4 != 0 || sr >= (int64_t(1) << 36)) return false;
  return (reinterpret_cast<uintptr_t>(base + distinct[0]) & 15) == 0;
}

// How many two-CTA clusters of the pair kernel fit on the device at once (queried once per context).
static int pair_slots(pai_ctx* ctx) {
  if (ctx->gemm_pair_slots == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (ctx->sm_count / 2));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = GemmShape<true>::kBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (smem_limit(ctx, k_gemm_tc<true>, GemmShape<true>::kBytes) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, k_gemm_tc<true>, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = -1;  // the pair kernel is not used on this device
    }
    ctx->gemm_pair_slots = n;
  }
  return ctx->gemm_pair_slots;
}

static pai_status launch_gemm(pai_ctx* ctx, const GemmArgs& g, bool pair, const PairMaps& maps) {
  const int total = g.tiles_m * g.tiles_n * g.batches * g.splits;
  KernelTimerScope timer(ctx, "gemm", 2.0 * g.m * g.n * (double)g.k_elems * g.batches);
  if (pair) {
    PAI_CUDA(smem_limit(ctx, k_gemm_tc<true>, GemmShape<true>::kBytes));
    const int pairs = std::min(total, pair_slots(ctx));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = GemmShape<true>::kBytes;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PAI_PDL_LAUNCH(cudaLaunchKernelEx(&cfg, k_gemm_tc<true>, g, maps), "tcgen05 gemm (CTA pairs)");
  } else {
    PAI_CUDA(smem_limit(ctx, k_gemm_tc<false>, GemmShape<false>::kBytes));
    const int grid = std::min(total, ctx->sm_count);
    k_gemm_tc<false><<<grid, kGemmThreads, GemmShape<false>::kBytes, ctx->stream>>>(g, maps);
    PAI_LAUNCH_CHECK("tcgen05 gemm");
  }
  return PAI_OK;
}

// Packs one operand (batched 2-D view) into hi/lo tiles.
// Allocates the packed hi/lo planes of one operand (batched 2-D view) and fills its pack descriptor; `doff` holds
// the batch offsets when there are more than fit inline and must outlive the launch.
static pai_status prepare_pack(pai_ctx* ctx, const float* base, const std::vector<int64_t>& boffs, int64_t sr, int64_t sk,
                               int rows, int k, int rt_pad, bool lo_only, Scratch* hi, Scratch* lo, Scratch* doff,
                               PackDesc* out) {
  int kt = (k + kBK - 1) / kBK;
  size_t floats = (size_t)boffs.size() * kt * rt_pad * kTileFloats;
  if (!lo_only) PAI_TRY(scratch(ctx, floats * 4, hi));
  PAI_TRY(scratch(ctx, floats * 4, lo));
  if (boffs.size() > (size_t)kInlineBatches) PAI_TRY(upload(ctx, boffs.data(), boffs.size() * 8, doff));
  // 16-byte loads along the unit-stride axis: every batch matrix and row start 16-byte aligned, and the unit-stride
  // extent a multiple of 4 so a vector never crosses the edge.
  bool aligned = (reinterpret_cast<uintptr_t>(base) & 15) == 0;
  for (int64_t o : boffs) aligned = aligned && (o % 4 == 0);
  int vec = 0;
  if (aligned && sk == 1 && sr % 4 == 0 && k % 4 == 0) vec = 1;
  else if (aligned && sr == 1 && sk % 4 == 0 && rows % 4 == 0) vec = 1;
  PackDesc d{};
  d.src = base;
  d.batch_off = static_cast<const int64_t*>(doff->p);
  if (!d.batch_off)
    for (size_t i = 0; i < boffs.size(); i++) d.boff_inline[i] = boffs[i];
  d.sr = sr; d.sk = sk; d.rows = rows; d.k = k; d.kt = kt; d.rt_pad = rt_pad; d.vec = vec; d.lo_only = lo_only ? 1 : 0;
  *out = d;
  return PAI_OK;
}

// Packs both operands of a product with one launch (k_pack), the operand with fewer tiles first.
static pai_status pack_operands(pai_ctx* ctx, const PackDesc& da, int batches_a, const Scratch& ahi, const Scratch& alo,
                                const PackDesc& db, int batches_b, const Scratch& bhi, const Scratch& blo) {
  const int64_t ta = (int64_t)da.kt * da.rt_pad * batches_a, tb = (int64_t)db.kt * db.rt_pad * batches_b;
  const bool b_first = tb <= ta;
  PackPair p{};
  p.d[0] = b_first ? db : da;
  p.d[1] = b_first ? da : db;
  p.hi[0] = static_cast<float*>(b_first ? bhi.p : ahi.p);
  p.lo[0] = static_cast<float*>(b_first ? blo.p : alo.p);
  p.hi[1] = static_cast<float*>(b_first ? ahi.p : bhi.p);
  p.lo[1] = static_cast<float*>(b_first ? alo.p : blo.p);
  p.tiles0 = b_first ? tb : ta;
  const int64_t total = ta + tb;
  if (total <= 0) return PAI_OK;
  if (total > INT32_MAX) return set_error(PAI_ERR_UNSUPPORTED, "MatMul: %lld operand tiles exceed one launch", (long long)total);
  k_pack<<<(unsigned)total, 256, 0, ctx->stream>>>(p);
  PAI_LAUNCH_CHECK("gemm pack");
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_matmul(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, int32_t tb, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, a, "a"));
  PAI_TRY(check_view(ctx, b, "b"));
  int ra = a->rank, rb = b->rank;
  if (ra < 2 || rb < 2)
    return set_error(PAI_ERR_ARGUMENT, "MatMul requires rank >= 2 operands; got %s and %s.", shape_str(*a).c_str(),
                     shape_str(*b).c_str());
  int m = a->dims[ra - 2], k = a->dims[ra - 1];
  int kb = tb ? b->dims[rb - 1] : b->dims[rb - 2];
  int n = tb ? b->dims[rb - 2] : b->dims[rb - 1];
  if (k != kb)
    return set_error(PAI_ERR_ARGUMENT, "MatMul inner dimensions disagree: %s x %s (transposeB=%s).", shape_str(*a).c_str(),
                     shape_str(*b).c_str(), tb ? "True" : "False");
  pai_tensor abt{}, bbt{};
  abt.rank = ra - 2;
  bbt.rank = rb - 2;
  for (int i = 0; i < abt.rank; i++) abt.dims[i] = a->dims[i];
  for (int i = 0; i < bbt.rank; i++) bbt.dims[i] = b->dims[i];
  int brank;
  int32_t bdims[PAI_MAX_RANK];
  if (!broadcast_shape(abt, bbt, &brank, bdims) || brank + 2 > PAI_MAX_RANK)
    return set_error(PAI_ERR_ARGUMENT, "Shapes %s and %s are not broadcast-compatible.", shape_str(abt).c_str(),
                     shape_str(bbt).c_str());
  int32_t od[PAI_MAX_RANK];
  for (int i = 0; i < brank; i++) od[i] = bdims[i];
  od[brank] = m;
  od[brank + 1] = n;
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, brank + 2, od, a->dtype, false, &r));
  int64_t batch = 1;
  for (int i = 0; i < brank; i++) batch *= bdims[i];
  if (batch == 0 || m == 0 || n == 0) { *out = r; return PAI_OK; }
  if (k == 0) {
    PAI_CUDA(cudaMemsetAsync(r.base, 0, (size_t)numel(r) * 4, ctx->stream));
    *out = r;
    return PAI_OK;
  }

  // Per output batch: the element offset of the A and B matrices (size-1 batch dims repeat, CpuComputeBackend.cs:222-233),
  // and the index of the distinct A / B batch matrices so each is packed once.
  std::vector<int64_t> a_off((size_t)batch), b_off((size_t)batch);
  std::vector<int32_t> a_idx((size_t)batch), b_idx((size_t)batch);
  std::vector<int64_t> a_distinct, b_distinct;
  {
    int64_t na = 1, nb = 1;
    for (int i = 0; i < abt.rank; i++) na *= abt.dims[i];
    for (int i = 0; i < bbt.rank; i++) nb *= bbt.dims[i];
    a_distinct.resize((size_t)na);
    b_distinct.resize((size_t)nb);
    // offsets of the distinct batch matrices, row-major over each operand's own batch dims
    for (int64_t i = 0; i < na; i++) {
      int64_t rem = i, off = a->offset;
      for (int d = abt.rank - 1; d >= 0; d--) { off += (rem % abt.dims[d]) * a->strides[d]; rem /= abt.dims[d]; }
      a_distinct[(size_t)i] = off;
    }
    for (int64_t i = 0; i < nb; i++) {
      int64_t rem = i, off = b->offset;
      for (int d = bbt.rank - 1; d >= 0; d--) { off += (rem % bbt.dims[d]) * b->strides[d]; rem /= bbt.dims[d]; }
      b_distinct[(size_t)i] = off;
    }
    std::vector<int> counter((size_t)brank, 0);
    for (int64_t bi = 0; bi < batch; bi++) {
      int64_t ia = 0, ib = 0;
      int la = brank - abt.rank, lb = brank - bbt.rank;
      for (int i = 0; i < abt.rank; i++) ia = ia * abt.dims[i] + (abt.dims[i] == 1 ? 0 : counter[(size_t)(la + i)]);
      for (int i = 0; i < bbt.rank; i++) ib = ib * bbt.dims[i] + (bbt.dims[i] == 1 ? 0 : counter[(size_t)(lb + i)]);
      a_idx[(size_t)bi] = (int32_t)ia;
      b_idx[(size_t)bi] = (int32_t)ib;
      a_off[(size_t)bi] = a_distinct[(size_t)ia];
      b_off[(size_t)bi] = b_distinct[(size_t)ib];
      for (int ax = brank - 1; ax >= 0; ax--) {
        if (++counter[(size_t)ax] < bdims[ax]) break;
        counter[(size_t)ax] = 0;
      }
    }
  }
  int64_t sam = a->strides[ra - 2], sak = a->strides[ra - 1];
  int64_t sbn = tb ? b->strides[rb - 2] : b->strides[rb - 1];
  int64_t sbk = tb ? b->strides[rb - 1] : b->strides[rb - 2];
  const float* abase = static_cast<const float*>(a->base);
  const float* bbase = static_cast<const float*>(b->base);

  // Decode-sized x · Wᵀ (at most 32 rows against one weight matrix): weight-streaming kernel (gemv.cu).
  const int64_t rows_total = batch * (int64_t)m;
  if (tb && b_distinct.size() == 1 && rows_total <= 32 && sak == 1 && sbk == 1) {
    int64_t xo[32];
    int idx = 0;
    for (int64_t bi = 0; bi < batch; bi++)
      for (int i = 0; i < m; i++) xo[idx++] = a_off[(size_t)bi] + (int64_t)i * sam;
    PAI_TRY(gemv_tn(ctx, abase, xo, (int)rows_total, bbase + b_distinct[0], sbn, n, k, fptr(r)));
    *out = r;
    return PAI_OK;
  }

  int kt = (k + kBK - 1) / kBK;
  int mt = (m + kBM - 1) / kBM;
  const int tn = (n + kTileN - 1) / kTileN;
  // Tile shape by the rounds the persistent CTAs take: 128 x 256 tiles on every SM, or 256 x 256 tiles on two-SM
  // clusters (same work per SM and round, but each SM reads half of B per MMA, which shared-memory bandwidth limits
  // in the one-CTA kernel to ~0.8 of the tensor pipe). Split-K products (few tiles, deep K) stay on one CTA each.
  const int64_t tiles1 = (int64_t)mt * tn * batch;
  const int64_t tiles2 = (int64_t)((m + 255) / 256) * tn * batch;
  int splits = 1;
  if (tiles1 * 2 <= ctx->sm_count && kt >= 16) {
    splits = ctx->sm_count / (int)tiles1;
    if (splits > kt / 8) splits = kt / 8;
    if (splits < 1) splits = 1;
  }
  int kt_per_split = (kt + splits - 1) / splits;
  splits = (kt + kt_per_split - 1) / kt_per_split;
  bool pair = false;
  if (splits == 1 && m > kBM) {
    const int slots = pair_slots(ctx);
    if (slots > 0) {
      const double rounds1 = std::ceil((double)tiles1 / ctx->sm_count) / 0.8;
      const double rounds2 = std::ceil((double)tiles2 / slots) * ((double)ctx->sm_count / (2.0 * slots)) / 0.95;
      pair = rounds2 < rounds1;
    }
  }
  const int mt_pad = pair ? 2 * (int)((m + 255) / 256) : mt;
  const int nt_pad = tn * (kTileN / kBM);
  const int64_t arows = (int64_t)a_distinct.size() * kt * mt_pad * kBM, brows = (int64_t)b_distinct.size() * kt * nt_pad * kBM;
  if (pair && (arows > INT32_MAX || brows > INT32_MAX))
    pair = false;  // tensor-map coordinates are 32-bit; the packed A (pairs of row tiles) serves the one-CTA kernel too
  // Pair kernel: a K-major operand's hi is the operand itself, so its pack writes lo alone.
  const bool a_raw = pair && raw_operand_ok(abase, a_distinct, sam, sak, k);
  const bool b_raw = pair && raw_operand_ok(bbase, b_distinct, sbn, sbk, k);
  Scratch ahi, alo, bhi, blo, dai, dbi, part;
  Scratch aoff, boff;
  PackDesc pda, pdb;
  PAI_TRY(prepare_pack(ctx, abase, a_distinct, sam, sak, m, k, mt_pad, a_raw, &ahi, &alo, &aoff, &pda));
  PAI_TRY(prepare_pack(ctx, bbase, b_distinct, sbn, sbk, n, k, nt_pad, b_raw, &bhi, &blo, &boff, &pdb));
  PAI_TRY(pack_operands(ctx, pda, (int)a_distinct.size(), ahi, alo, pdb, (int)b_distinct.size(), bhi, blo));
  if (batch > kInlineBatches) {
    PAI_TRY(upload(ctx, a_idx.data(), a_idx.size() * 4, &dai));
    PAI_TRY(upload(ctx, b_idx.data(), b_idx.size() * 4, &dbi));
  }
  float* cdst = fptr(r);
  if (splits > 1) {
    PAI_TRY(scratch(ctx, (size_t)splits * numel(r) * 4, &part));
    cdst = static_cast<float*>(part.p);
  }
  GemmArgs g{};
  g.a_hi = static_cast<float*>(ahi.p); g.a_lo = static_cast<float*>(alo.p);
  g.b_hi = static_cast<float*>(bhi.p); g.b_lo = static_cast<float*>(blo.p);
  g.a_index = static_cast<int32_t*>(dai.p); g.b_index = static_cast<int32_t*>(dbi.p);
  if (batch <= kInlineBatches)
    for (int64_t i = 0; i < batch; i++) { g.a_index_inline[i] = a_idx[(size_t)i]; g.b_index_inline[i] = b_idx[(size_t)i]; }
  g.c = cdst; g.m = m; g.n = n; g.kt = kt; g.mt_pad = mt_pad; g.nt_pad = nt_pad;
  g.tiles_m = pair ? mt_pad / 2 : mt; g.tiles_n = tn; g.batches = (int)batch; g.splits = splits;
  g.kt_per_split = kt_per_split;
  g.error_flag = ctx->d_error_flag;
  g.k_elems = k;
  g.a_raw = a_raw ? 1 : 0;
  g.b_raw = b_raw ? 1 : 0;
  PairMaps maps;
  memset(&maps, 0, sizeof maps);
  if (pair) {
    if (a_raw) PAI_TRY(raw_map(abase + a_distinct[0], m, k, sam, &maps.a_hi));
    else PAI_TRY(plane_map(g.a_hi, arows, &maps.a_hi));
    PAI_TRY(plane_map(g.a_lo, arows, &maps.a_lo));
    if (b_raw) PAI_TRY(raw_map(bbase + b_distinct[0], n, k, sbn, &maps.b_hi));
    else PAI_TRY(plane_map(g.b_hi, brows, &maps.b_hi));
    PAI_TRY(plane_map(g.b_lo, brows, &maps.b_lo));
  }
  PAI_TRY(launch_gemm(ctx, g, pair, maps));
  if (splits > 1) {
    int64_t nn = numel(r);
    k_splitk_reduce<<<grid_for(ctx, nn, 256), 256, 0, ctx->stream>>>(cdst, fptr(r), nn, splits);
    PAI_LAUNCH_CHECK("splitk reduce");
  }
  *out = r;
  return PAI_OK;
}

// Reads and clears the device error flag that bounded waits in the kernels report into.
PAI_API pai_status pai_check_device_error(pai_ctx* ctx, int32_t* code) {
  PAI_TRY(enter(ctx));
  int v = 0;
  PAI_CUDA(cudaMemcpyAsync(&v, ctx->d_error_flag, 4, cudaMemcpyDeviceToHost, ctx->stream));
  PAI_CUDA(cudaStreamSynchronize(ctx->stream));
  if (v) PAI_CUDA(cudaMemsetAsync(ctx->d_error_flag, 0, 4, ctx->stream));
  if (code) *code = v;
  if (v) return set_error(PAI_ERR_TIMEOUT, "a kernel wait timed out (site %d); results of the affected launch are invalid", v);
  return PAI_OK;
}
