// Tensor-core (tcgen05, 3xTF32) fused causal attention backward.
//
// The gradients of the composed chain of Modules.cs:169-203 under the Autograd rules (MatMul Autograd.cs:54-73,
// Softmax :197-205, Mul by the 1/√d scale :39-47, GQA group sum ReduceGradToShape :320-333):
//   P = exp(S − lse), dP = dO·Vᵀ, dS = P ⊙ (dP − rowsum(dO ⊙ O)),
//   dV = Σ_group Pᵀ·dO,  dK = Σ_group dSᵀ·(q·scale),  dQ = scale · dS·K.
//
// Two kernels of 384 threads (bulk-copy producers, warps 2-9 element-wise — two warps per TMEM lane quadrant, 32 of
// each 64-wide block's columns per thread — and MMA issuers, one thread each, every one consuming its own ring or
// barrier: one thread issues a tf32 MMA about every 115 cycles whatever its N, and the tensor pipe overlaps several
// threads' N=64 products):
//   k_attn_bwd_kv_tc  128 keys of one (batch, kv head) stay resident (K, V as A operands in shared memory); the
//                     group's heads x 64-query blocks stream through two rings of half tiles, q·scale and dO for the
//                     score issuer, dOᵀ and (q·scale)ᵀ for the gradient issuer; Sᵀ and dPᵀ land in TMEM, Pᵀ / dSᵀ go
//                     back to TMEM as hi/lo A operands of dV += Pᵀ·dO and dK += dSᵀ·(q·scale).
//   k_attn_bwd_q_tc   128 queries of one (batch, head) stay resident: q·scale in shared memory, dO in TMEM (so dP is
//                     a TS product). 64-key blocks stream through per-operand rings (two K and two V slots, so a
//                     block's K and V land while the previous block's products run; one Kᵀ slot, a block behind);
//                     dS goes to TMEM as the A operand of dQ += dS·K.
// All operands are 64-row SWIZZLE_128B hi/lo tiles from k_attn_pack; 128-row A operands are assembled in shared
// memory from two 64-row tiles. Every wait is bounded (device error flag on timeout).
// Accuracy: the gradient products of each streamed block go into a fresh TMEM accumulator, which the element-wise
// warps add into fp32 registers (IEEE round-to-nearest) before the next block's products overwrite it: the tensor
// core's own accumulation over the hundreds of blocks a long sequence streams (x the GQA group) drifts from the
// float64 result far more than a rounded fp32 sum does.
#include <math.h>

#include "common.cuh"
#include "tc_common.cuh"
#include "attention_pack.cuh"

namespace pai {

using namespace tc;

namespace bwd {

constexpr int kRows = 128;               // resident rows per CTA (keys or queries)
constexpr int kBlk = 64;                 // streamed block (queries or keys)
constexpr int kDP = 64;                  // padded head dim
constexpr uint32_t kTile = 64 * 64 * 4 * 2;   // one packed 64x64 hi/lo tile: 32 KB
constexpr uint32_t kA = 2 * kTile;            // a resident 128-row operand: 64 KB
// Both kernels: 224 KB of operands (dK/dV: resident K and V + two rings of three half tiles; dQ: resident q·scale +
// five tile slots), then the alignment slack and the barriers.
constexpr int kSmem = 2 * kA + 3 * kTile + 1024 + 256;
constexpr uint32_t kTmemCols = 512;

struct Args {
  const float* qs;   // q·scale, 64-row tiles   [B*H][nq2][tile]
  const float* dO;   // dO,      64-row tiles   [B*H][nq2][tile]
  const float* qsT;  // (q·scale)ᵀ tiles        [B*H][nq][tile]
  const float* dOT;  // dOᵀ tiles               [B*H][nq][tile]
  const float* k;    // k, 64-row tiles         [B*KVH][nk2][tile]
  const float* v;    // v, 64-row tiles         [B*KVH][nk2][tile]
  const float* kT;   // kᵀ tiles                [B*KVH][nk][tile]
  const float* lse;  // [B,H,S]
  const float* dvec; // [B,H,S]  rowsum(dO ⊙ O)
  float* dq;         // [B,H,S,D]
  float* dk;         // [B,KVH,L,D]
  float* dv;         // [B,KVH,L,D]
  int B, H, KVH, S, L, D, pos_offset, causal;
  int nq, nq2, nk, nk2;  // 64-blocks along S and L (nq2/nk2 rounded up to even)
  float scale;
  int* error_flag;
};

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Resident 128-row operand from two consecutive 64-row packed tiles: smem (hl, kb) sub-tile = 16 KB, rows 64-127 at +8 KB.
__device__ __forceinline__ void load_resident(uint8_t* dst, const float* tile0, uint64_t* bar) {
#pragma unroll
  for (int half = 0; half < 2; half++)
#pragma unroll
    for (int hk = 0; hk < 4; hk++)  // (hl, kb) in the packed order hi kb0, hi kb1, lo kb0, lo kb1
      bulk_g2s(dst + hk * 16384 + half * 8192, tile0 + (size_t)half * (kTile / 4) + (size_t)hk * 2048, 8192, bar);
}

// S(+)= A(128-row resident, smem) · B(64-row tile, smem)ᵀ over the padded head dim.
__device__ __forceinline__ void mma_res_tile(uint32_t d, uint32_t a, uint32_t bt, uint32_t idesc) {
  const uint32_t a_lo = a + kA / 2, b_lo = bt + kTile / 2;
#pragma unroll
  for (int ks = 0; ks < kDP / 8; ks++) {
    uint32_t ao = (ks >> 2) * 16384 + (ks & 3) * 32, bo = (ks >> 2) * 8192 + (ks & 3) * 32;
    mma_ss(d, desc_sw128(a_lo + ao), desc_sw128(bt + bo), idesc, ks > 0 ? 1u : 0u);
    mma_ss(d, desc_sw128(a + ao), desc_sw128(b_lo + bo), idesc, 1u);
    mma_ss(d, desc_sw128(a + ao), desc_sw128(bt + bo), idesc, 1u);
  }
}

// D(+)= A(TMEM hi/lo, 64 columns of K) · B(64-row tile over the same K)ᵀ
__device__ __forceinline__ void mma_tmem_tile(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t bt, uint32_t idesc,
                                              bool accumulate) {
  const uint32_t b_lo = bt + kTile / 2;
#pragma unroll
  for (int ks = 0; ks < kBlk / 8; ks++) {
    uint32_t bo = (ks >> 2) * 8192 + (ks & 3) * 32;
    uint32_t c = (uint32_t)(ks * 8);
    mma_ts(d, a_lo + c, desc_sw128(bt + bo), idesc, (accumulate || ks > 0) ? 1u : 0u);
    mma_ts(d, a_hi + c, desc_sw128(b_lo + bo), idesc, 1u);
    mma_ts(d, a_hi + c, desc_sw128(bt + bo), idesc, 1u);
  }
}

// The dK/dV kernel streams each block's four tiles through two rings of half-tile slots, each with its own producer
// thread and its own issuing thread (so every ring has one consumer, which takes its slots in load order): the score
// ring carries q·scale then dO (the Sᵀ and dPᵀ products), the gradient ring dOᵀ then (q·scale)ᵀ (dV and dK). A half
// is one 32-wide half of the tile's K: its hi and lo 64 x 32 sub-tiles, 16 KB, released once the 12 MMAs that read
// it complete, so the next tile streams in while the second half's MMAs run.
constexpr uint32_t kHalf = kTile / 2;
constexpr int kHalfSlots = 3;

// Item j of a block (0-1: first tile's halves, 2-3: second tile's) of packed tile `tile` into a half slot.
__device__ __forceinline__ void load_half(uint8_t* dst, const float* tile, int half, uint64_t* bar) {
  mbar_expect_tx(bar, kHalf);
  bulk_g2s(dst, tile + half * 2048, 8192, bar);            // hi, K columns [32*half, 32*half + 32)
  bulk_g2s(dst + 8192, tile + (2 + half) * 2048, 8192, bar);  // lo
}

// One ring of kHalfSlots half-tile slots, consumed in order by one thread; item i sits in slot i % kHalfSlots.
struct HalfRing {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  __device__ __forceinline__ uint32_t slot_addr(int i) const { return smem_u32(base + (i % kHalfSlots) * kHalf); }
  __device__ __forceinline__ bool wait_full(int i) const { return mbar_wait(&full[i % kHalfSlots], (uint32_t)(i / kHalfSlots) & 1u); }
  __device__ __forceinline__ uint64_t* empty_of(int i) const { return &empty[i % kHalfSlots]; }
};

// S(+)= A(128-row resident, smem) · B(tile in ring items i, i+1)ᵀ; each half's slot is released after its MMAs.
__device__ __forceinline__ bool mma_res_halves(uint32_t d, uint32_t a, const HalfRing& r, int i, uint32_t idesc) {
  const uint32_t a_lo = a + kA / 2;
#pragma unroll
  for (int hf = 0; hf < 2; hf++) {
    if (!r.wait_full(i + hf)) return false;
    fence_after();
    const uint32_t bh = r.slot_addr(i + hf), bl = bh + 8192;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const int ks = 4 * hf + kk;
      const uint32_t ao = (ks >> 2) * 16384 + kk * 32, bo = kk * 32;
      mma_ss(d, desc_sw128(a_lo + ao), desc_sw128(bh + bo), idesc, ks > 0 ? 1u : 0u);
      mma_ss(d, desc_sw128(a + ao), desc_sw128(bl + bo), idesc, 1u);
      mma_ss(d, desc_sw128(a + ao), desc_sw128(bh + bo), idesc, 1u);
    }
    commit(r.empty_of(i + hf));
  }
  return true;
}

// D = A(TMEM hi/lo, 64 columns of K) · B(tile in ring items i, i+1)ᵀ; each half's slot is released after its MMAs.
__device__ __forceinline__ bool mma_tmem_halves(uint32_t d, uint32_t a_hi, uint32_t a_lo, const HalfRing& r, int i,
                                                uint32_t idesc) {
#pragma unroll
  for (int hf = 0; hf < 2; hf++) {
    if (!r.wait_full(i + hf)) return false;
    fence_after();
    const uint32_t bh = r.slot_addr(i + hf), bl = bh + 8192;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const int ks = 4 * hf + kk;
      const uint32_t c = (uint32_t)(ks * 8), bo = kk * 32;
      mma_ts(d, a_lo + c, desc_sw128(bh + bo), idesc, ks > 0 ? 1u : 0u);
      mma_ts(d, a_hi + c, desc_sw128(bl + bo), idesc, 1u);
      mma_ts(d, a_hi + c, desc_sw128(bh + bo), idesc, 1u);
    }
    commit(r.empty_of(i + hf));
  }
  return true;
}

// 32 values -> TMEM as tf32 hi/lo, 8 columns at a time (the element-wise warps keep their block's scores and both
// gradient accumulators in registers meanwhile).
__device__ __forceinline__ void store_hilo(uint32_t hi_addr, uint32_t lo_addr, const float* x) {
#pragma unroll
  for (int h = 0; h < 4; h++) {
    float hi[8], lo[8];
#pragma unroll
    for (int c = 0; c < 8; c++) split_tf32_fast(x[8 * h + c], hi[c], lo[c]);
    tmem_st8(hi_addr + 8 * h, hi);
    tmem_st8(lo_addr + 8 * h, lo);
  }
}

// acc += 32 TMEM columns of this warp's lanes (one block's partial gradient rows), 8 at a time.
__device__ __forceinline__ void add_partial(uint32_t taddr, float* acc) {
#pragma unroll
  for (int h = 0; h < 4; h++) {
    float v[8];
    tmem_ld8(taddr + 8 * h, v);
#pragma unroll
    for (int c = 0; c < 8; c++) acc[8 * h + c] += v[c];
  }
}

// ---------------------------------------------------------------- dK, dV
// dK/dV kernel roles (12 warps): 0 score-ring producer (and the resident K, V), 1 score issuer (Sᵀ, dPᵀ; TMEM owner),
// 2-9 element-wise, 10 gradient issuer (dV, dK), 11 gradient-ring producer.
constexpr int kScoreProducerKV = 0, kGradIssuerKV = 10, kGradProducerKV = 11;
constexpr int kThreadsKV = 32 * (kGradProducerKV + 1);

__global__ void __launch_bounds__(kThreadsKV, 1) k_attn_bwd_kv_tc(Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + kA;
  uint8_t* sScore = smem + 2 * kA;                 // score ring: kHalfSlots half tiles
  uint8_t* sGrad = sScore + kHalfSlots * kHalf;    // gradient ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGrad + kHalfSlots * kHalf);
  uint64_t* a_full = bars;
  uint64_t* sc_full = bars + 1;     // [3]
  uint64_t* sc_empty = bars + 4;    // [3]
  uint64_t* gr_full = bars + 7;     // [3]
  uint64_t* gr_empty = bars + 10;   // [3]
  uint64_t* st_full = bars + 13;
  uint64_t* st_free = bars + 14;
  uint64_t* pd_full = bars + 15;
  uint64_t* pd_free = bars + 16;
  uint64_t* drained = bars + 17;    // [2]: each issuer's MMAs have completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // key tiles in the slowest grid index: under a causal mask tile 0 is attended by every query, so the longest
  // tiles start first (ordered by (batch, kv head) instead, the CTAs read 5x less from DRAM but the longest tiles of
  // the last heads started last and the backward took 15% longer in the 1B step)
  const int kt = blockIdx.z, kvh = blockIdx.x, b = blockIdx.y;
  const int g = a.H / a.KVH;
  const int j0 = kt * kRows;
  int qb_start = 0;
  if (a.causal) {
    int first = j0 - a.pos_offset;  // the first query that can see key j0
    qb_start = first > 0 ? first / kBlk : 0;
  }
  const int qb_count = a.nq > qb_start ? a.nq - qb_start : 0;
  const int N = g * qb_count;  // (head, query block) pairs streamed past these keys
  // TMEM columns
  const uint32_t cS = 0, cDP = 64, cPhi = 128, cPlo = 192, cDShi = 256, cDSlo = 320, cDV = 384, cDK = 448;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int i = 0; i < kHalfSlots; i++) {
      mbar_init(&sc_full[i], 1); mbar_init(&sc_empty[i], 1);
      mbar_init(&gr_full[i], 1); mbar_init(&gr_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_free, 8);
    mbar_init(pd_full, 8);
    mbar_init(pd_free, 1);
    for (int i = 0; i < 2; i++) mbar_init(&drained[i], 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const HalfRing score{sScore, sc_full, sc_empty}, grad{sGrad, gr_full, gr_empty};

  auto head_of = [&](int n) { return kvh * g + n / max(qb_count, 1); };
  auto qblk_of = [&](int n) { return qb_start + n % max(qb_count, 1); };

  if (warp == kScoreProducerKV || warp == kGradProducerKV) {
    if (lane == 0 && N > 0) {
      const bool sc = warp == kScoreProducerKV;
      const HalfRing& r = sc ? score : grad;
      if (sc) {
        size_t kvbase = ((size_t)(b * a.KVH + kvh) * a.nk2 + 2 * kt) * (kTile / 4);
        mbar_expect_tx(a_full, 2 * kA);
        load_resident(sK, a.k + kvbase, a_full);
        load_resident(sV, a.v + kvbase, a_full);
      }
      // per block: items 0-1 the halves of q·scale (score) / dOᵀ (gradient), items 2-3 of dO / (q·scale)ᵀ
      for (int i = 0; i < 4 * N && !s_abort; i++) {
        const int n = i >> 2, j = i & 3;
        if (!mbar_wait(r.empty_of(i), ((uint32_t)(i / kHalfSlots) & 1u) ^ 1u)) {
          atomicCAS(a.error_flag, 0, sc ? 21 : 23);
          s_abort = 1;
          break;
        }
        const size_t bh = (size_t)(b * a.H + head_of(n));
        const int qb = qblk_of(n);
        const float* tile = sc ? (j < 2 ? a.qs : a.dO) + (bh * a.nq2 + qb) * (kTile / 4)
                               : (j < 2 ? a.dOT : a.qsT) + (bh * a.nq + qb) * (kTile / 4);
        load_half(r.base + (i % kHalfSlots) * kHalf, tile, j & 1, &r.full[i % kHalfSlots]);
      }
      // every half copied has been consumed before the CTA may exit
      for (int i = 4 * N; i < 4 * N + kHalfSlots; i++)
        mbar_wait(r.empty_of(i), ((uint32_t)(i / kHalfSlots) & 1u) ^ 1u);
    }
  } else if (warp == 1 || warp == kGradIssuerKV) {
    if (lane == 0 && N > 0) {
      constexpr uint32_t idesc = idesc_tf32(128, 64);
      const int role = warp == 1 ? 0 : 1;
      bool ok = true;
      if (role == 0) {
        ok = mbar_wait(a_full, 0);
        for (int n = 0; n < N && ok && !s_abort; n++) {
          if (n > 0 && !mbar_wait(st_free, (n - 1) & 1)) { ok = false; break; }
          ok = mma_res_halves(tmem + cS, smem_u32(sK), score, 4 * n, idesc) &&        // Sᵀ  = K·(q·scale)ᵀ
               mma_res_halves(tmem + cDP, smem_u32(sV), score, 4 * n + 2, idesc);     // dPᵀ = V·dOᵀ
          if (ok) commit(st_full);
        }
      } else {
        for (int n = 0; n < N && ok && !s_abort; n++) {
          if (!mbar_wait(pd_full, n & 1)) { ok = false; break; }
          fence_after();
          ok = mma_tmem_halves(tmem + cDV, tmem + cPhi, tmem + cPlo, grad, 4 * n, idesc) &&        // dV_n = Pᵀ·dO
               mma_tmem_halves(tmem + cDK, tmem + cDShi, tmem + cDSlo, grad, 4 * n + 2, idesc);    // dK_n = dSᵀ·qs
          if (ok) commit(pd_free);
        }
      }
      if (!ok) { atomicCAS(a.error_flag, 0, 22 + 2 * role); s_abort = 1; }
      // every MMA this thread issued completes before the CTA releases its tensor memory
      commit(&drained[role]);
      mbar_wait(&drained[role], 0);
    }
  } else if (warp >= 2 && warp < 10) {
    const int sw = warp - 2, quad = warp & 3, half = sw >> 2;
    const int row = quad * 32 + lane;
    const int key = j0 + row;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t col = (uint32_t)(32 * half);
    const float kLog2e = 1.4426950408889634f;
    bool ok = N > 0;
    float dvv[32], dkk[32];  // this thread's dV, dK row slice, summed block by block in fp32
#pragma unroll
    for (int d = 0; d < 32; d++) { dvv[d] = 0.0f; dkk[d] = 0.0f; }
    for (int n = 0; n < N; n++) {
      const int h = head_of(n), q0 = qblk_of(n) * kBlk + (int)col;
      // the block's 32 query statistics: one load per lane, issued before the wait, broadcast by shuffles below
      const int ql = q0 + lane;
      const float lse_l = ql < a.S ? a.lse[((int64_t)b * a.H + h) * a.S + ql] * kLog2e : 0.0f;
      const float dv_l = ql < a.S ? a.dvec[((int64_t)b * a.H + h) * a.S + ql] : 0.0f;
      float s[32], dp[32];
#pragma unroll
      for (int c = 0; c < 32; c++) { s[c] = 0.0f; dp[c] = 0.0f; }
      if (ok && !warp_wait(st_full, n & 1)) { ok = false; if (lane == 0) atomicCAS(a.error_flag, 0, 26 + 0); }
      if (ok) {
        fence_after();
        tmem_ld32(tmem + lane_off + cS + col, s);
        tmem_ld32(tmem + lane_off + cDP + col, dp);
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(st_free);
      }
#pragma unroll
      for (int c = 0; c < 32; c++) {
        int q = q0 + c;
        const float lse2 = __shfl_sync(0xffffffffu, lse_l, c);
        const float dvc = __shfl_sync(0xffffffffu, dv_l, c);
        bool vis = q < a.S && key < a.L && (!a.causal || key <= a.pos_offset + q);
        float p = vis ? ex2_sfu(fmaf(s[c], kLog2e, -lse2)) : 0.0f;
        float dvq = vis ? dvc : 0.0f;
        s[c] = p;
        dp[c] = p * (dp[c] - dvq);
      }
      if (ok && n > 0 && !warp_wait(pd_free, (n - 1) & 1)) { ok = false; if (lane == 0) atomicCAS(a.error_flag, 0, 26 + 1); }
      if (ok && n > 0) {
        // block n-1's products are done: fold them in before block n's P / dS (and then its products) reuse TMEM
        fence_after();
        add_partial(tmem + lane_off + cDV + col, dvv);
        add_partial(tmem + lane_off + cDK + col, dkk);
      }
      if (ok) {
        store_hilo(tmem + lane_off + cPhi + col, tmem + lane_off + cPlo + col, s);
        store_hilo(tmem + lane_off + cDShi + col, tmem + lane_off + cDSlo + col, dp);
        tmem_st_wait();
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pd_full);
      }
    }
    if (ok && N > 0 && !warp_wait(pd_free, (N - 1) & 1)) { ok = false; if (lane == 0) atomicCAS(a.error_flag, 0, 26 + 2); }
    if (ok || N == 0) {
      // keys that no query sees (N == 0) get zero gradients: every output row is written
      if (N > 0) {
        fence_after();
        add_partial(tmem + lane_off + cDV + col, dvv);
        add_partial(tmem + lane_off + cDK + col, dkk);
      }
      if (key < a.L) {
        int64_t base = (((int64_t)b * a.KVH + kvh) * a.L + key) * a.D;
#pragma unroll
        for (int d = 0; d < 32; d++)
          if ((int)col + d < a.D) { a.dv[base + col + d] = dvv[d]; a.dk[base + col + d] = dkk[d]; }
      }
    }
    if (!ok && N > 0 && lane == 0) s_abort = 1;
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- dQ
// dQ kernel roles (12 warps): 0 producer, 1 S issuer (and TMEM owner), 2-9 element-wise, 10 dP issuer, 11 dQ issuer.
constexpr int kDpWarpQ = 10, kDqWarpQ = 11;
constexpr int kThreadsQ = 32 * (kDqWarpQ + 1);

__global__ void __launch_bounds__(kThreadsQ, 1) k_attn_bwd_q_tc(Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // q·scale stays in shared memory (A of S = (q·scale)·Kᵀ); dO stays in TMEM (A of dP = dO·Vᵀ), which leaves room for
  // two K and two V slots, so each block's K and V land while the previous block's products run.
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kA;              // [2]
  uint8_t* sV = sK + 2 * kTile;         // [2]
  uint8_t* sKT = sV + 2 * kTile;        // [1]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKT + kTile);
  uint64_t* a_full = bars;
  uint64_t* k_full = bars + 1;      // [2]
  uint64_t* k_empty = bars + 3;     // [2]
  uint64_t* v_full = bars + 5;      // [2]
  uint64_t* v_empty = bars + 7;     // [2]
  uint64_t* kt_full = bars + 9;
  uint64_t* kt_empty = bars + 10;
  uint64_t* do_ready = bars + 11;   // dO is in TMEM
  uint64_t* st_full = bars + 12;
  uint64_t* st_free = bars + 13;
  uint64_t* pd_full = bars + 14;
  uint64_t* pd_free = bars + 15;
  uint64_t* drained = bars + 16;    // [3]: each issuer's MMAs have completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = (int)gridDim.z - 1 - (int)blockIdx.z;  // query tiles slowest and reversed: longest causal tiles first
  const int h = blockIdx.x, b = blockIdx.y;
  const int kvh = h / (a.H / a.KVH);
  const int q0 = qt * kRows;
  int kend = a.L;
  if (a.causal) kend = min(a.L, a.pos_offset + q0 + kRows);
  const int N = kend > 0 ? (kend + kBlk - 1) / kBlk : 0;
  const uint32_t cS = 0, cDP = 64, cDShi = 128, cDSlo = 192, cDQ = 256, cDOhi = 320, cDOlo = 384;
  const size_t qbase = ((size_t)(b * a.H + h) * a.nq2 + 2 * qt) * (kTile / 4);

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1);
    }
    mbar_init(kt_full, 1);
    mbar_init(kt_empty, 1);
    mbar_init(do_ready, 8);
    mbar_init(st_full, 2);   // the S and dP issuers
    mbar_init(st_free, 8);
    mbar_init(pd_full, 8);
    mbar_init(pd_free, 1);
    for (int i = 0; i < 3; i++) mbar_init(&drained[i], 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && N > 0) {
      mbar_expect_tx(a_full, kA);
      load_resident(sQ, a.qs + qbase, a_full);
      const size_t kv = (size_t)(b * a.KVH + kvh);
      // One tile into a slot once its previous fill is released (fill f waits for parity (f & 1) ^ 1).
      auto load = [&](uint64_t* empty, int fill, uint64_t* full, uint8_t* dst, const float* src) -> bool {
        if (!mbar_wait(empty, (uint32_t)(fill & 1) ^ 1u)) { atomicCAS(a.error_flag, 0, 31); s_abort = 1; return false; }
        mbar_expect_tx(full, kTile);
        bulk_g2s(dst, src, kTile, full);
        return true;
      };
      // K_n and V_n, then Kᵀ_{n-1}: the dQ product of a block runs a block behind its scores, so its tile trails
      // and never holds up the next block's K and V.
      bool ok = true;
      for (int n = 0; n <= N && ok && !s_abort; n++) {
        if (n < N) {
          const int sl = n & 1;
          ok = load(&k_empty[sl], n >> 1, &k_full[sl], sK + sl * kTile, a.k + (kv * a.nk2 + n) * (kTile / 4)) &&
               load(&v_empty[sl], n >> 1, &v_full[sl], sV + sl * kTile, a.v + (kv * a.nk2 + n) * (kTile / 4));
        }
        if (ok && n >= 1) ok = load(kt_empty, n - 1, kt_full, sKT, a.kT + (kv * a.nk + (n - 1)) * (kTile / 4));
      }
      // every tile copied has been consumed before the CTA may exit
      for (int sl = 0; sl < 2; sl++) {
        const int fills = (N - sl + 1) / 2;
        mbar_wait(&k_empty[sl], (uint32_t)(fills & 1) ^ 1u);
        mbar_wait(&v_empty[sl], (uint32_t)(fills & 1) ^ 1u);
      }
      mbar_wait(kt_empty, (uint32_t)(N & 1) ^ 1u);
    }
  } else if (warp == 1 || warp == kDpWarpQ || warp == kDqWarpQ) {
    const int role = warp == 1 ? 0 : (warp == kDpWarpQ ? 1 : 2);  // 0 S, 1 dP, 2 dQ: one ring or barrier each
    if (lane == 0 && N > 0) {
      constexpr uint32_t idesc = idesc_tf32(128, 64);
      bool ok = true;
      if (role < 2) {
        ok = mbar_wait(role == 0 ? a_full : do_ready, 0);
        uint64_t* full = role == 0 ? k_full : v_full;
        uint64_t* empty = role == 0 ? k_empty : v_empty;
        for (int n = 0; n < N && ok && !s_abort; n++) {
          const int sl = n & 1;
          if (n > 0 && !mbar_wait(st_free, (n - 1) & 1)) { ok = false; break; }
          if (!mbar_wait(&full[sl], (n >> 1) & 1)) { ok = false; break; }
          fence_after();
          if (role == 0)
            mma_res_tile(tmem + cS, smem_u32(sQ), smem_u32(sK + sl * kTile), idesc);  // S = (q·scale)·Kᵀ
          else
            mma_tmem_tile(tmem + cDP, tmem + cDOhi, tmem + cDOlo, smem_u32(sV + sl * kTile), idesc, false);  // dO·Vᵀ
          commit(st_full);
          commit(&empty[sl]);
        }
      } else {
        for (int n = 0; n < N && ok && !s_abort; n++) {
          if (!mbar_wait(pd_full, n & 1) || !mbar_wait(kt_full, n & 1)) { ok = false; break; }
          fence_after();
          mma_tmem_tile(tmem + cDQ, tmem + cDShi, tmem + cDSlo, smem_u32(sKT), idesc, false);  // dQ_n = dS·K
          commit(pd_free);
          commit(kt_empty);
        }
      }
      if (!ok) { atomicCAS(a.error_flag, 0, 32 + role); s_abort = 1; }
      commit(&drained[role]);
      mbar_wait(&drained[role], 0);
    }
  } else if (warp >= 2 && warp < 10) {
    const int sw = warp - 2, quad = warp & 3, half = sw >> 2;
    const int row = quad * 32 + lane;
    const int qi = q0 + row;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t col = (uint32_t)(32 * half);
    const float kLog2e = 1.4426950408889634f;
    const float lse2 = qi < a.S ? a.lse[((int64_t)b * a.H + h) * a.S + qi] * kLog2e : 0.0f;
    const float dvq = qi < a.S ? a.dvec[((int64_t)b * a.H + h) * a.S + qi] : 0.0f;
    bool ok = N > 0;
    if (N > 0) {
      // This thread's dO row slice (packed hi/lo, 32 columns) -> TMEM, the A operand of the dP products. In the packed
      // 64-row tile the (hi|lo, column half) sub-tile is 64 rows of 32 floats with 16-byte chunks XOR (row & 7).
      const float* t = a.dO + qbase + (size_t)(row >> 6) * (kTile / 4);
      const int rr = row & 63;
      float hv[32], lv[32];
#pragma unroll
      for (int c4 = 0; c4 < 8; c4++) {
        const int off = rr * 32 + ((c4 ^ (rr & 7)) << 2);
        const float4 x = *reinterpret_cast<const float4*>(t + half * 2048 + off);
        const float4 y = *reinterpret_cast<const float4*>(t + (2 + half) * 2048 + off);
        hv[4 * c4] = x.x; hv[4 * c4 + 1] = x.y; hv[4 * c4 + 2] = x.z; hv[4 * c4 + 3] = x.w;
        lv[4 * c4] = y.x; lv[4 * c4 + 1] = y.y; lv[4 * c4 + 2] = y.z; lv[4 * c4 + 3] = y.w;
      }
      tmem_st32(tmem + lane_off + cDOhi + col, hv);
      tmem_st32(tmem + lane_off + cDOlo + col, lv);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(do_ready);
    }
    float dq[32];  // this thread's dQ row slice, summed block by block in fp32
#pragma unroll
    for (int d = 0; d < 32; d++) dq[d] = 0.0f;
    for (int n = 0; n < N; n++) {
      float s[32], dp[32];
#pragma unroll
      for (int c = 0; c < 32; c++) { s[c] = 0.0f; dp[c] = 0.0f; }
      if (ok && !warp_wait(st_full, n & 1)) { ok = false; if (lane == 0) atomicCAS(a.error_flag, 0, 36 + 0); }
      if (ok) {
        fence_after();
        tmem_ld32(tmem + lane_off + cS + col, s);
        tmem_ld32(tmem + lane_off + cDP + col, dp);
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(st_free);
      }
      const int k0 = n * kBlk + (int)col;
#pragma unroll
      for (int c = 0; c < 32; c++) {
        int kj = k0 + c;
        bool vis = qi < a.S && kj < a.L && (!a.causal || kj <= a.pos_offset + qi);
        float p = vis ? ex2_sfu(fmaf(s[c], kLog2e, -lse2)) : 0.0f;
        dp[c] = p * (dp[c] - dvq);
      }
      if (ok && n > 0 && !warp_wait(pd_free, (n - 1) & 1)) { ok = false; if (lane == 0) atomicCAS(a.error_flag, 0, 36 + 1); }
      if (ok && n > 0) {
        fence_after();
        add_partial(tmem + lane_off + cDQ + col, dq);  // block n-1's dS·K, before block n's dS and product
      }
      if (ok) {
        store_hilo(tmem + lane_off + cDShi + col, tmem + lane_off + cDSlo + col, dp);
        tmem_st_wait();
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pd_full);
      }
    }
    if (ok && N > 0 && !warp_wait(pd_free, (N - 1) & 1)) { ok = false; if (lane == 0) atomicCAS(a.error_flag, 0, 36 + 2); }
    if (ok || N == 0) {
      // queries that see no key (N == 0) get zero gradients: every output row is written
      if (N > 0) {
        fence_after();
        add_partial(tmem + lane_off + cDQ + col, dq);
      }
      if (qi < a.S) {
        int64_t base = (((int64_t)b * a.H + h) * a.S + qi) * a.D;
#pragma unroll
        for (int d = 0; d < 32; d++)
          if ((int)col + d < a.D) a.dq[base + col + d] = dq[d] * a.scale;
      }
    }
    if (!ok && N > 0 && lane == 0) s_abort = 1;
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace bwd

}  // namespace pai

using namespace pai;

// Backward on the tensor cores for head dims <= 64. dvec = rowsum(dO ⊙ O) [B,H,S] (already computed).
pai_status attn_tc_bwd(pai_ctx* ctx, const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, const pai_tensor& dout,
                       const float* lse, const float* dvec, int B, int H, int KVH, int S, int L, int D, float scale,
                       int causal, int pos_offset, float* dq, float* dk, float* dv) {
  using namespace bwd;
  int nq = (S + kBlk - 1) / kBlk, nk = (L + kBlk - 1) / kBlk;
  int nq2 = (nq + 1) & ~1, nk2 = (nk + 1) & ~1;
  size_t tf = kTile;
  Scratch qs, dO, qsT, dOT, kp, vp, kT;
  PAI_TRY(scratch(ctx, (size_t)B * H * nq2 * tf, &qs));
  PAI_TRY(scratch(ctx, (size_t)B * H * nq2 * tf, &dO));
  PAI_TRY(scratch(ctx, (size_t)B * H * nq * tf, &qsT));
  PAI_TRY(scratch(ctx, (size_t)B * H * nq * tf, &dOT));
  PAI_TRY(scratch(ctx, (size_t)B * KVH * nk2 * tf, &kp));
  PAI_TRY(scratch(ctx, (size_t)B * KVH * nk2 * tf, &vp));
  PAI_TRY(scratch(ctx, (size_t)B * KVH * nk * tf, &kT));
  // [B, X, R, D] view strides of each operand (dout is [B,S,H,D]: its head axis is 2, its row axis 1).
  AttnPackArgs packs[kAttnPackMax];
  int npack = 0;
  auto pack = [&](const float* base, int64_t sb, int64_t sx, int64_t sr, int64_t sd, int X, int R, int transpose,
                  float sc, int nblk, void* dst) -> pai_status {
    if (npack == kAttnPackMax) return set_error(PAI_ERR_ARGUMENT, "attention backward: too many packed operands");
    packs[npack++] = AttnPackArgs{base, sb, sx, sr, sd, X, R, D, kBlk, transpose, sc, nblk, static_cast<float*>(dst)};
    return PAI_OK;
  };
  const float* qb = static_cast<const float*>(q.base) + q.offset;
  const float* kb = static_cast<const float*>(k.base) + k.offset;
  const float* vb = static_cast<const float*>(v.base) + v.offset;
  const float* ob = static_cast<const float*>(dout.base) + dout.offset;
  PAI_TRY(pack(qb, q.strides[0], q.strides[1], q.strides[2], q.strides[3], H, S, 0, scale, nq2, qs.p));
  PAI_TRY(pack(qb, q.strides[0], q.strides[1], q.strides[2], q.strides[3], H, S, 1, scale, nq, qsT.p));
  PAI_TRY(pack(ob, dout.strides[0], dout.strides[2], dout.strides[1], dout.strides[3], H, S, 0, 1.0f, nq2, dO.p));
  PAI_TRY(pack(ob, dout.strides[0], dout.strides[2], dout.strides[1], dout.strides[3], H, S, 1, 1.0f, nq, dOT.p));
  PAI_TRY(pack(kb, k.strides[0], k.strides[1], k.strides[2], k.strides[3], KVH, L, 0, 1.0f, nk2, kp.p));
  PAI_TRY(pack(kb, k.strides[0], k.strides[1], k.strides[2], k.strides[3], KVH, L, 1, 1.0f, nk, kT.p));
  PAI_TRY(pack(vb, v.strides[0], v.strides[1], v.strides[2], v.strides[3], KVH, L, 0, 1.0f, nk2, vp.p));
  PAI_TRY(attn_pack_launch(ctx, packs, npack, B));  // all seven operands in one launch
  PAI_CUDA(smem_limit(ctx, k_attn_bwd_kv_tc, kSmem));
  PAI_CUDA(smem_limit(ctx, k_attn_bwd_q_tc, kSmem));
  Args args{static_cast<float*>(qs.p), static_cast<float*>(dO.p), static_cast<float*>(qsT.p), static_cast<float*>(dOT.p),
            static_cast<float*>(kp.p), static_cast<float*>(vp.p), static_cast<float*>(kT.p), lse, dvec, dq, dk, dv,
            B, H, KVH, S, L, D, pos_offset, causal, nq, nq2, nk, nk2, scale, ctx->d_error_flag};
  dim3 gkv((unsigned)KVH, (unsigned)B, (unsigned)((L + kRows - 1) / kRows));
  k_attn_bwd_kv_tc<<<gkv, kThreadsKV, kSmem, ctx->stream>>>(args);
  PAI_LAUNCH_CHECK("attention bwd dK/dV (tcgen05)");
  dim3 gq((unsigned)H, (unsigned)B, (unsigned)((S + kRows - 1) / kRows));
  k_attn_bwd_q_tc<<<gq, kThreadsQ, kSmem, ctx->stream>>>(args);
  PAI_LAUNCH_CHECK("attention bwd dQ (tcgen05)");
  return PAI_OK;
}
