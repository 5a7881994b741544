// Tensor-core (tcgen05, 3xTF32) fused causal attention forward.
//
// Semantics of the composed chain of Modules.cs:169-203 (entry point pai_sdpa_fwd in attention.cu):
// scores = (q·scale)·kᵀ with q rounded to fp32 after scaling, keys j <= pos_offset + i, online softmax, ·v, output in
// the merged-heads layout [B,S,H,D] plus the row log-sum-exp for the backward.
//
// Per work item: 128 queries of one (batch, head), key blocks of 64, head dim padded to 64; one persistent CTA per SM
// walks its items.
//   pre-pass k_attn_pack: q·scale, k and vᵀ split into tf32 hi/lo and written as SWIZZLE_128B K-major tiles;
//   warp 0      bulk-copies the Q tile once and K/Vᵀ blocks into a 2-stage ring;
//   warp 1      allocates TMEM and issues S = Q·Kᵀ (3 MMAs per k-step, M=128 N=64) into a double-buffered TMEM S;
//   warp 10     issues O_j = P_j·V_j with P read from TMEM as the A operand (a second issuing thread: one thread
//               issues a tf32 MMA about every 115 cycles whatever its N, and the pipe overlaps two threads' products);
//   warps 2-9   softmax: two warps per TMEM lane quadrant, so each query row is owned by two threads, each holding
//               32 of the block's 64 scores (and 32 of the 64 output columns); the pair agrees on the running row
//               max through shared memory. Each thread masks (diagonal blocks only), exponentiates, splits P into
//               hi/lo and stores it to TMEM, and accumulates its half of O_j in registers with the running rescale.
// Every wait is bounded; a timeout raises the context's device error flag and the CTA drains and exits.
#include <math.h>

#include "common.cuh"
#include "tc_common.cuh"
#include "attention_pack.cuh"

namespace pai {

using namespace tc;

constexpr int kQT = 128;  // queries per CTA
constexpr int kKB = 64;   // keys per block
constexpr int kDP = 64;   // padded head dim
constexpr int kSoftmaxWarps = 8;
constexpr int kPvWarp = 2 + kSoftmaxWarps;  // the P·V issuer, after the softmax warps
constexpr int kFwdThreads = 32 * (kPvWarp + 1);

// ---------------------------------------------------------------- pack pre-pass
// One tile (bi of the nblk along R) of one (batch, head) row bx of an operand. Output per tile: [hi kb0][hi kb1]
// [lo kb0][lo kb1], kb = 32 columns, rows x 32 floats each.
__device__ __forceinline__ void attn_pack_tile(const AttnPackArgs& a, int bi, int bx) {
  __shared__ float tile[kQT][kDP + 1];
  int b = bx / a.X, x = bx % a.X;
  const float* src = a.src + b * a.s_b + x * a.s_x;
  int rows = a.transpose ? kDP : a.blk;
  int p0 = bi * a.blk;
  // 16-byte loads along the head dim when it is unit-stride, every row start is 16-byte aligned and D % 4 == 0.
  bool vec = a.s_d == 1 && (a.D & 3) == 0 && (a.s_r & 3) == 0 && ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
  if (vec) {
    for (int idx = threadIdx.x; idx < a.blk * (kDP / 4); idx += blockDim.x) {
      int pos = idx / (kDP / 4), d = (idx % (kDP / 4)) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p0 + pos < a.R && d < a.D) {
        v = *reinterpret_cast<const float4*>(src + (int64_t)(p0 + pos) * a.s_r + d);
        if (a.scale != 1.0f) {
          v.x = __fmul_rn(v.x, a.scale); v.y = __fmul_rn(v.y, a.scale);
          v.z = __fmul_rn(v.z, a.scale); v.w = __fmul_rn(v.w, a.scale);
        }
      }
      if (a.transpose) {
        tile[d][pos] = v.x; tile[d + 1][pos] = v.y; tile[d + 2][pos] = v.z; tile[d + 3][pos] = v.w;
      } else {
        tile[pos][d] = v.x; tile[pos][d + 1] = v.y; tile[pos][d + 2] = v.z; tile[pos][d + 3] = v.w;
      }
    }
  }
  for (int idx = vec ? a.blk * kDP : threadIdx.x; idx < a.blk * kDP; idx += blockDim.x) {
    int pos = idx / kDP, d = idx % kDP;
    float v = 0.0f;
    if (p0 + pos < a.R && d < a.D) {
      v = src[(int64_t)(p0 + pos) * a.s_r + (int64_t)d * a.s_d];
      if (a.scale != 1.0f) v = __fmul_rn(v, a.scale);
    }
    if (a.transpose) tile[d][pos] = v;
    else tile[pos][d] = v;
  }
  __syncthreads();
  float* out = a.out + ((size_t)bx * a.nblk + bi) * (size_t)(4 * rows * 32);
  for (int ch = threadIdx.x; ch < 2 * rows * 8; ch += blockDim.x) {
    int kb = ch / (rows * 8), rem = ch % (rows * 8);
    int r = rem >> 3, c = rem & 7;
    float hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; j++) split_tf32(tile[r][kb * 32 + c * 4 + j], hi[j], lo[j]);
    int phys = r * 8 + (c ^ (r & 7));
    reinterpret_cast<float4*>(out + (size_t)kb * rows * 32)[phys] = make_float4(hi[0], hi[1], hi[2], hi[3]);
    reinterpret_cast<float4*>(out + (size_t)(2 + kb) * rows * 32)[phys] = make_float4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// Several operands in one launch: CTAs [start[i], start[i+1]) pack operand i, its tiles in (bx, bi) order.
struct AttnPackSet {
  AttnPackArgs p[kAttnPackMax];
  int64_t start[kAttnPackMax + 1];
  int n;
};

__global__ void __launch_bounds__(256) k_attn_pack(const __grid_constant__ AttnPackSet s) {
  const int64_t i = blockIdx.x;
  int k = 0;
#pragma unroll
  for (int j = 1; j < kAttnPackMax; j++)
    if (j < s.n && i >= s.start[j]) k = j;
  const AttnPackArgs& a = *(&s.p[0] + k);
  const int64_t local = i - *(&s.start[0] + k);
  attn_pack_tile(a, (int)(local % a.nblk), (int)(local / a.nblk));
}

pai_status attn_pack_launch(pai_ctx* ctx, const AttnPackArgs* packs, int n, int B) {
  if (n < 1 || n > kAttnPackMax) return set_error(PAI_ERR_ARGUMENT, "attention pack: %d operands (1..%d)", n, kAttnPackMax);
  AttnPackSet s{};
  int64_t total = 0;
  for (int i = 0; i < n; i++) {
    s.p[i] = packs[i];
    s.start[i] = total;
    total += (int64_t)packs[i].nblk * B * packs[i].X;
  }
  s.start[n] = total;
  s.n = n;
  if (total > INT32_MAX) return set_error(PAI_ERR_UNSUPPORTED, "attention pack: %lld tiles exceed one launch", (long long)total);
  if (total > 0) {
    k_attn_pack<<<(unsigned)total, 256, 0, ctx->stream>>>(s);
    PAI_LAUNCH_CHECK("attention pack");
  }
  return PAI_OK;
}

// ---------------------------------------------------------------- forward kernel
struct AttnTcArgs {
  const float* qp;  // [B*H][q_tiles][64 KB]
  const float* kp;  // [B*KVH][k_blocks][32 KB]
  const float* vp;  // [B*KVH][k_blocks][32 KB]  (vᵀ tiles)
  float* out;       // [B,S,H,D]
  float* lse;       // [B,H,S]
  int B, H, KVH, S, L, D, pos_offset, causal, q_tiles, k_blocks;
  int* error_flag;
};

constexpr uint32_t kQBytes = kQT * kDP * 4 * 2;        // 64 KB (hi + lo)
constexpr uint32_t kKBytes = kKB * kDP * 4 * 2;        // 32 KB
// K and Vᵀ blocks travel in separate rings: a K slot frees as soon as S = Q·Kᵀ of its block is done, a Vᵀ slot after
// P·V, so the next blocks' loads start a block earlier than with one ring of (K, Vᵀ) stages.
constexpr int kKStages = 2, kVStages = 2;
constexpr int kFwdSmemBytes = kQBytes + (kKStages + kVStages) * kKBytes + 1024 + 256;
// TMEM columns
// TMEM columns: S double buffer, then two slots of (P hi, P lo, P·V): P of block j and the product P_j·V_j use slot
// j & 1, so the softmax warps write P_{j+1} while P_j·V_j is still being computed.
constexpr uint32_t kColS0 = 0, kColS1 = 64, kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_phi(int slot) { return 128u + 192u * (uint32_t)slot; }
__host__ __device__ constexpr uint32_t col_plo(int slot) { return 192u + 192u * (uint32_t)slot; }
__host__ __device__ constexpr uint32_t col_pv(int slot) { return 256u + 192u * (uint32_t)slot; }

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// One work item: a 128-query tile of one (batch, head).
struct FwdItem {
  int qt, h, b, kvh, q0, nblk;
};

// Item t in longest-first order (the query tile slowest and reversed, then head, then batch); false when the tile
// sees no key. (Ordering the items by (batch, kv head) groups instead cut the K/V reads from DRAM from 2.0 to 0.5 GB
// at [4, 32, 2048, 64] but lengthened the kernel, 0.63 -> 0.72 ms: the rounds then mix long and short tiles.)
__device__ __forceinline__ bool fwd_item(const AttnTcArgs& a, int t, FwdItem& it) {
  const int hb = a.H * a.B;
  it.qt = a.q_tiles - 1 - t / hb;
  const int rem = t % hb;
  it.h = rem % a.H;
  it.b = rem / a.H;
  it.kvh = it.h / (a.H / a.KVH);
  it.q0 = it.qt * kQT;
  int kend = a.L;
  if (a.causal) kend = min(a.L, a.pos_offset + it.q0 + kQT);
  it.nblk = kend > 0 ? (kend + kKB - 1) / kKB : 0;
  return it.nblk > 0;
}

// This CTA's next item from round r on: rounds are bands of gridDim.x consecutive items, walked forward in even
// rounds and backward in odd ones (CTA c takes band position c, then gridDim.x - 1 - c), so a CTA that drew a long
// tile in one band draws a short one in the next. Returns false when the CTA has no further item; r is left at the
// round of the item returned.
__device__ __forceinline__ bool next_fwd_item(const AttnTcArgs& a, int n_items, int& r, FwdItem& it) {
  const int G = gridDim.x, c = blockIdx.x;
  for (; r * G < n_items; r++) {
    const int t = r * G + ((r & 1) ? G - 1 - c : c);
    if (t < n_items && fwd_item(a, t, it)) return true;
  }
  return false;
}

// Persistent: one CTA per SM walks its items (next_fwd_item). Barrier phases, ring slots and TMEM slots follow a
// running block counter J over the CTA's items, so a tile's last blocks and the next tile's first loads overlap: the
// next K block is fetched while this tile finishes, and the next Q tile as soon as this tile's last S product has
// read Q (q_empty).
__global__ void __launch_bounds__(kFwdThreads, 1) k_attn_fwd_tc(AttnTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kQBytes;                 // [kKStages] K hi/lo blocks
  uint8_t* sV = sK + kKStages * kKBytes;        // [kVStages] Vᵀ hi/lo blocks
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kVStages * kKBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;                     // [kKStages]
  uint64_t* k_empty = k_full + kKStages;           // [kKStages]
  uint64_t* v_full = k_empty + kKStages;           // [kVStages]
  uint64_t* v_empty = v_full + kVStages;           // [kVStages]
  uint64_t* s_full = v_empty + kVStages;           // [2]
  uint64_t* s_free = s_full + 2;                   // [2]
  uint64_t* p_full = s_free + 2;                   // [2]
  uint64_t* pv_full = p_full + 2;                  // [2]
  uint64_t* drained = pv_full + 2;                 // [2]: the S and P·V issuers' MMAs have completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 2);
  __shared__ volatile int s_abort;
  __shared__ float s_max[2][2][kQT];  // [block parity][column half][row]
  __shared__ float s_l[2][kQT];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = a.q_tiles * a.H * a.B;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < kKStages; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; i++) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kSoftmaxWarps);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&p_full[i], kSoftmaxWarps);
      mbar_init(&pv_full[i], 1);
      mbar_init(&drained[i], 1);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // loads in the order the MMA warp consumes them: K of the first block, then per block the next block's K
      // (possibly the next tile's first) before this block's Vᵀ; each tile's Q once the previous tile's S products
      // are done with the Q buffer
      auto load_k = [&](int J, const FwdItem& it, int j) {
        const int st = J % kKStages;
        if (!mbar_wait(&k_empty[st], ((J / kKStages) & 1) ^ 1)) return false;
        const size_t head_off = (size_t)(it.b * a.KVH + it.kvh) * a.k_blocks;
        mbar_expect_tx(&k_full[st], kKBytes);
        bulk_g2s(sK + st * kKBytes, a.kp + (head_off + j) * (kKBytes / 4), kKBytes, &k_full[st]);
        return true;
      };
      auto load_v = [&](int J, const FwdItem& it, int j) {
        const int st = J % kVStages;
        if (!mbar_wait(&v_empty[st], ((J / kVStages) & 1) ^ 1)) return false;
        const size_t head_off = (size_t)(it.b * a.KVH + it.kvh) * a.k_blocks;
        mbar_expect_tx(&v_full[st], kKBytes);
        bulk_g2s(sV + st * kKBytes, a.vp + (head_off + j) * (kKBytes / 4), kKBytes, &v_full[st]);
        return true;
      };
      int r = 0, J0 = 0, ord = 0;
      FwdItem cur;
      bool have = next_fwd_item(a, n_items, r, cur);
      bool ok = !have || load_k(0, cur, 0);
      while (have && ok && !s_abort) {
        if (ord > 0 && !mbar_wait(q_empty, (ord - 1) & 1)) { ok = false; break; }
        mbar_expect_tx(q_full, kQBytes);
        bulk_g2s(sQ, a.qp + ((size_t)(cur.b * a.H + cur.h) * a.q_tiles + cur.qt) * (kQBytes / 4), kQBytes, q_full);
        int rn = r + 1;
        FwdItem nxt;
        const bool have_next = next_fwd_item(a, n_items, rn, nxt);
        for (int j = 0; j < cur.nblk && ok && !s_abort; j++) {
          const int J = J0 + j;
          if (j + 1 < cur.nblk) ok = load_k(J + 1, cur, j + 1);
          else if (have_next) ok = load_k(J + 1, nxt, 0);
          if (ok) ok = load_v(J, cur, j);
        }
        J0 += cur.nblk;
        ord++;
        cur = nxt;
        r = rn;
        have = have_next;
      }
      if (!ok) { atomicExch(a.error_flag, 11); s_abort = 1; }
      // drain: every issued load must land (and be consumed) before the CTA exits
      for (int J = J0; J < J0 + kKStages; J++) mbar_wait(&k_empty[J % kKStages], ((J / kKStages) & 1) ^ 1);
      for (int J = J0; J < J0 + kVStages; J++) mbar_wait(&v_empty[J % kVStages], ((J / kVStages) & 1) ^ 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(128, 64);
      const uint32_t q_hi = smem_u32(sQ), q_lo = q_hi + kQBytes / 2;
      // S_J = Q·K_Jᵀ into S slot J & 1, once K_J has landed and the softmax warps have read S_{J-2} from that slot
      auto wait_s = [&](int J) {
        return mbar_wait(&k_full[J % kKStages], (J / kKStages) & 1) && mbar_wait(&s_free[J & 1], ((J >> 1) & 1) ^ 1);
      };
      auto issue_s = [&](int J) {
        const int st = J & 1;
        uint32_t k_hi = smem_u32(sK + (J % kKStages) * kKBytes), k_lo = k_hi + kKBytes / 2;
        uint32_t d = tmem + (st ? kColS1 : kColS0);
#pragma unroll
        for (int ks = 0; ks < kDP / 8; ks++) {
          uint32_t qo = (ks >> 2) * (kQT * 128) + (ks & 3) * 32;  // Q kb stride 16 KB
          uint32_t ko = (ks >> 2) * (kKB * 128) + (ks & 3) * 32;  // K kb stride 8 KB
          mma_ss(d, desc_sw128(q_lo + qo), desc_sw128(k_hi + ko), idesc, ks > 0 ? 1u : 0u);
          mma_ss(d, desc_sw128(q_hi + qo), desc_sw128(k_lo + ko), idesc, 1u);
          mma_ss(d, desc_sw128(q_hi + qo), desc_sw128(k_hi + ko), idesc, 1u);
        }
        commit(&s_full[st]);
        commit(&k_empty[J % kKStages]);  // the K block is free once these MMAs have read it
      };
      int r = 0, J0 = 0, ord = 0;
      FwdItem it;
      bool ok = true;
      while (ok && !s_abort && next_fwd_item(a, n_items, r, it)) {
        if (!mbar_wait(q_full, ord & 1)) { atomicExch(a.error_flag, 12); s_abort = 1; break; }
        for (int j = 0; j < it.nblk; j++) {
          const int J = J0 + j;
          if (!wait_s(J)) { atomicExch(a.error_flag, 13); s_abort = 1; ok = false; break; }
          fence_after();
          issue_s(J);
          if (j + 1 == it.nblk) commit(q_empty);  // this tile's S products are all issued: Q may be replaced after them
        }
        J0 += it.nblk;
        ord++;
        r++;
      }
      // every MMA this thread issued completes before the CTA releases its tensor memory
      commit(&drained[0]);
      mbar_wait(&drained[0], 0);
    }
  } else if (warp == kPvWarp) {
    // O_J = P_J·V_J, issued by a second thread: one thread issues a tcgen05.mma about every 115 cycles whatever its
    // N, and the tensor pipe runs two threads' N=64 products side by side, so S and P·V no longer queue behind
    // each other
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(128, 64);
      int r = 0, J0 = 0;
      FwdItem it;
      bool ok = true;
      while (ok && !s_abort && next_fwd_item(a, n_items, r, it)) {
        for (int j = 0; j < it.nblk; j++) {
          const int J = J0 + j;
          const int ps = J & 1;  // P / P·V slot of this block
          const int vs = J % kVStages;
          if (!mbar_wait(&p_full[ps], (J >> 1) & 1) || !mbar_wait(&v_full[vs], (J / kVStages) & 1)) {
            atomicExch(a.error_flag, 14); s_abort = 1; ok = false; break;
          }
          fence_after();
          uint32_t v_hi = smem_u32(sV + vs * kKBytes), v_lo = v_hi + kKBytes / 2;
          uint32_t d = tmem + col_pv(ps);
#pragma unroll
          for (int ks = 0; ks < kKB / 8; ks++) {
            uint32_t vo = (ks >> 2) * (kDP * 128) + (ks & 3) * 32;  // Vᵀ kb (32 keys) stride 8 KB
            uint32_t pc = (uint32_t)(ks * 8);
            mma_ts(d, tmem + col_plo(ps) + pc, desc_sw128(v_hi + vo), idesc, ks > 0 ? 1u : 0u);
            mma_ts(d, tmem + col_phi(ps) + pc, desc_sw128(v_lo + vo), idesc, 1u);
            mma_ts(d, tmem + col_phi(ps) + pc, desc_sw128(v_hi + vo), idesc, 1u);
          }
          commit(&pv_full[ps]);
          commit(&v_empty[vs]);
        }
        J0 += it.nblk;
        r++;
      }
      commit(&drained[1]);
      mbar_wait(&drained[1], 0);
    }
  } else if (warp < 2 + kSoftmaxWarps) {
    // softmax warps: (quad, half) -> query row quad*32+lane, columns [32*half, 32*half+32) of S, P and O
    const int sw = warp - 2;
    const int quad = warp & 3;
    const int half = sw >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t col = (uint32_t)(32 * half);
    const float kLog2e = 1.4426950408889634f;
    // After a timed-out wait `ok` turns false for good: the warp skips all further TMEM and barrier work but still
    // reaches every named barrier, so its partner warp never waits on it.
    bool ok = true;
    int r = 0, J0 = 0;
    FwdItem it;
    while (next_fwd_item(a, n_items, r, it)) {
      const int q0 = it.q0, nblk = it.nblk;
      const int qi = q0 + row;
      float o[32];
#pragma unroll
      for (int d = 0; d < 32; d++) o[d] = 0.0f;
      float m = -INFINITY, l = 0.0f, alpha_prev = 1.0f;
      for (int j = 0; j < nblk; j++) {
        const int J = J0 + j;
        const int st = J & 1;
        float s[32];
#pragma unroll
        for (int c = 0; c < 32; c++) s[c] = 0.0f;
        if (ok && !warp_wait(&s_full[st], (J >> 1) & 1)) ok = false;
        if (ok) {
          fence_after();
          tmem_ld32(tmem + lane_off + (st ? kColS1 : kColS0) + col, s);
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[st]);
        }
        const int k0 = j * kKB;
        // Masking is needed only where the block crosses the causal diagonal or the end of the keys.
        const bool need_mask = (k0 + kKB > a.L) || (a.causal && k0 + kKB - 1 > a.pos_offset + q0);
        float mx = -INFINITY;
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < 32; c++) {
            int kj = k0 + (int)col + c;
            bool vis = kj < a.L && (!a.causal || kj <= a.pos_offset + qi);
            if (!vis) s[c] = -INFINITY;
            mx = fmaxf(mx, s[c]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; c++) mx = fmaxf(mx, s[c]);
        }
        // The row max over both halves: exchange through shared memory with the partner warp of this quadrant.
        s_max[st][half][row] = mx;
        named_sync(1 + quad, 64);
        mx = fmaxf(mx, s_max[st][half ^ 1][row]);
        float mn = fmaxf(m, mx);
        float alpha = (m == -INFINITY) ? 0.0f : __expf(m - mn);
        if (mn == -INFINITY) alpha = 1.0f;
        // A masked score (-inf) gives 2^-inf = 0; a row with no visible key yet keeps a zero bias, so no NaN forms.
        const float mn2 = (mn == -INFINITY) ? 0.0f : mn * kLog2e;
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int c = 0; c < 32; c++) {
          float p = ex2_sfu(fmaf(s[c], kLog2e, -mn2));
          s[c] = p;
          part[c & 3] += p;
        }
        const float sum = (part[0] + part[1]) + (part[2] + part[3]);
        l = l * alpha + sum;
        m = mn;
        // o holds the blocks up to j-3 in units of the running max. P_{j-2}·V_{j-2} (units of m_{j-2}) sits in this
        // block's slot: fold it in (factor exp(m_{j-2} - m_j) = alpha_{j-1}·alpha_j) before P_j takes the slot.
        const int ps = J & 1;
#pragma unroll
        for (int d = 0; d < 32; d++) o[d] *= alpha;
        if (ok && j >= 2) {
          if (!warp_wait(&pv_full[ps], ((J - 2) >> 1) & 1)) {
            ok = false;
          } else {
            fence_after();
            float pv[32];
            tmem_ld32(tmem + lane_off + col_pv(ps) + col, pv);
            const float f = alpha_prev * alpha;
#pragma unroll
            for (int d = 0; d < 32; d++) o[d] = fmaf(pv[d], f, o[d]);
          }
        }
        alpha_prev = alpha;
        if (ok) {
          // P_j -> TMEM as hi/lo (the A operand of P·V)
          float hi[32], lo[32];
#pragma unroll
          for (int c = 0; c < 32; c++) split_tf32_fast(s[c], hi[c], lo[c]);
          tmem_st32(tmem + lane_off + col_phi(ps) + col, hi);
          tmem_st32(tmem + lane_off + col_plo(ps) + col, lo);
          tmem_st_wait();
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[ps]);
        }
      }
      // the last two blocks' P·V products: P_{n-2}·V_{n-2} (units of m_{n-2}: factor alpha_{n-1}) and P_{n-1}·V_{n-1}
      for (int jj = (nblk >= 2 ? nblk - 2 : 0); ok && jj < nblk; jj++) {
        const int Jj = J0 + jj;
        const int ps = Jj & 1;
        if (!warp_wait(&pv_full[ps], (Jj >> 1) & 1)) {
          ok = false;
          break;
        }
        fence_after();
        float pv[32];
        tmem_ld32(tmem + lane_off + col_pv(ps) + col, pv);
        const float f = (jj == nblk - 1) ? 1.0f : alpha_prev;
#pragma unroll
        for (int d = 0; d < 32; d++) o[d] = fmaf(pv[d], f, o[d]);
      }
      s_l[half][row] = l;
      named_sync(1 + quad, 64);
      float lt = s_l[0][row] + s_l[1][row];
      if (ok && qi < a.S) {
        float inv = 1.0f / lt;
        float* orow = a.out + (((int64_t)it.b * a.S + qi) * a.H + it.h) * a.D;
#pragma unroll
        for (int d = 0; d < 32; d++)
          if ((int)col + d < a.D) orow[col + d] = o[d] * inv;
        if (half == 0) a.lse[((int64_t)it.b * a.H + it.h) * a.S + qi] = m + logf(lt);
      }
      J0 += nblk;
      r++;
    }
    if (!ok && lane == 0) { atomicExch(a.error_flag, 15); s_abort = 1; }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace pai

using namespace pai;

// Packs q (scaled), k and vᵀ and runs the tensor-core forward. Called by pai_sdpa_fwd for head dims <= 64.
pai_status attn_tc_fwd(pai_ctx* ctx, const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, int B, int H, int KVH,
                       int S, int L, int D, float scale, int causal, int pos_offset, float* out, float* lse) {
  int q_tiles = (S + kQT - 1) / kQT, k_blocks = (L + kKB - 1) / kKB;
  Scratch qp, kp, vp;
  PAI_TRY(scratch(ctx, (size_t)B * H * q_tiles * kQBytes, &qp));
  PAI_TRY(scratch(ctx, (size_t)B * KVH * k_blocks * kKBytes, &kp));
  PAI_TRY(scratch(ctx, (size_t)B * KVH * k_blocks * kKBytes, &vp));
  auto pack = [&](const pai_tensor& t, int X, int R, int blk, int transpose, float sc, int nblk, void* dst) {
    return AttnPackArgs{static_cast<const float*>(t.base) + t.offset, t.strides[0], t.strides[1], t.strides[2],
                        t.strides[3], X, R, D, blk, transpose, sc, nblk, static_cast<float*>(dst)};
  };
  const AttnPackArgs packs[3] = {pack(q, H, S, kQT, 0, scale, q_tiles, qp.p), pack(k, KVH, L, kKB, 0, 1.0f, k_blocks, kp.p),
                                 pack(v, KVH, L, kKB, 1, 1.0f, k_blocks, vp.p)};
  PAI_TRY(attn_pack_launch(ctx, packs, 3, B));
  PAI_CUDA(smem_limit(ctx, k_attn_fwd_tc, kFwdSmemBytes));
  AttnTcArgs args{static_cast<float*>(qp.p), static_cast<float*>(kp.p), static_cast<float*>(vp.p), out, lse,
                  B, H, KVH, S, L, D, pos_offset, causal, q_tiles, k_blocks, ctx->d_error_flag};
  const int n_items = q_tiles * H * B;
  const int grid = n_items < ctx->sm_count ? n_items : ctx->sm_count;  // persistent: one CTA per SM
  if (grid > 0) k_attn_fwd_tc<<<grid, kFwdThreads, kFwdSmemBytes, ctx->stream>>>(args);
  PAI_LAUNCH_CHECK("attention fwd (tcgen05)");
  return PAI_OK;
}
