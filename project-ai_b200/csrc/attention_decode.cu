// Attention for decode steps: a few query positions (S x g query rows per kv head, at most 16) against a long KV
// cache. Same result as the causal attention forward (Modules.cs:169-203: softmax(q·kᵀ·scale) · v, keys j visible
// to query row s when j <= pos_offset + s), computed in exact fp32 arithmetic.
//
// Decode attention reads every cached key and value once per step and does ~2 flops per byte, so it is bound by
// HBM, not by the tensor cores. One CTA per (key split, kv head, batch) holds all query rows of that kv head's group,
// so each K/V row is read from HBM once for all g heads that share it:
//   producer warp: one thread streams 16-key K and V tiles (contiguous rows: one bulk copy each) into an 8-stage
//                  shared-memory ring, so the CTA keeps up to 64 KB of loads in flight;
//   4 consumer warps: tile t goes to warp t % 4. QKᵀ: lanes l and l+16 split key l%16's head dims and read them
//                  in a lane-rotated order (no bank conflicts); online softmax per query row over the tile's 16
//                  lanes; PV: lanes own two head-dim elements, the tile's probabilities are read back as float4
//                  broadcasts from shared memory.
// The key splits of one (batch, kv head) form a thread-block cluster; they divide the visible keys [0, kend) evenly on
// the device (kend comes from the device-side position in a decode step), and cluster rank 0 merges the CTAs'
// partials through distributed shared memory. The 4 warps and then the splits are merged in a fixed order
// (log-sum-exp rescaling), so results are deterministic.
//
// Small batches (fewer than 64 (batch, kv head) pairs) leave each warp about one tile, too little for the ring to pay
// for itself: they take k_attn_decode_direct, in which every warp loads its own 32-key tile straight from global
// memory and which launches early behind the previous kernel. Both variants compute the same attention; they may
// round differently, and one shape always takes the same variant.
#include <cooperative_groups.h>
#include <math.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace pai {

namespace dec {

namespace cg = cooperative_groups;
using ::pai::tc::bulk_g2s;
using ::pai::tc::mbar_arrive;
using ::pai::tc::mbar_expect_tx;
using ::pai::tc::mbar_init;
using ::pai::tc::mbar_wait;
using ::pai::tc::warp_wait;

constexpr int kConsumers = 4;                      // consumer warps
constexpr int kThreads = 32 * (kConsumers + 1);    // + the producer warp
constexpr int kMaxD = 64;
constexpr int kMaxRows = 16;
constexpr int kTile = 16;                          // keys per tile
constexpr int kStages = 8;                         // ring depth: two tiles per consumer warp
static_assert(kStages % kConsumers == 0, "a stage must always belong to the same consumer warp");
constexpr int kHalfStage = kTile * kMaxD * 4;      // the K tile; the V tile follows it
constexpr int kStageBytes = 2 * kHalfStage;
constexpr size_t smem_bytes(int stages) { return (size_t)stages * kStageBytes + 2 * kStages * sizeof(uint64_t); }
constexpr int kMaxCluster = 8;                     // key splits of one (batch, kv head): a portable cluster
constexpr int kBarRope = 1;                        // named barrier: new cache rows written (consumers -> producer)
constexpr int kBarConsumers = 2;                   // named barrier among the consumer warps
constexpr int kDirectThreads = 128;                // latency variant (k_attn_decode_direct): 4 warps
constexpr int kDirectWarps = kDirectThreads / 32;
constexpr int kDirectTile = 32;                    // keys per warp step
constexpr int kDirectMinPairs = 64;                // the streaming kernel from this many (batch, kv head) pairs on

struct View {
  const float* p;
  int64_t s0, s1, s2;  // batch, head, position strides (head-dim stride is 1)
};

struct Args {
  View q, k, v;          // q [B,H,S,D]; k, v [B,KVH,L,D]
  int B, H, KVH, S, L, D, g, rows;
  int pos_offset, causal;
  float scale;
  int splits;            // CTAs per (batch, kv head): the cluster size along x
  int keys_per_split;    // latency variant: keys of each split (a multiple of 128)
  int stages;            // shared-memory ring depth (<= kStages): no deeper than the most tiles one CTA can get
  const float* pos_dev;  // when set: pos_offset = pos_dev[0] and the keys are cache positions 0 .. pos+S-1 (L = capacity)
  int* error_flag;
  // fused RoPE + cache append: q and the new key/value rows [B, KVH, S, D] arrive unrotated; keys are rotated with the
  // table rows pos + s and written with the values into the caches (k.p / v.p) before they are attended to
  View kn, vn;
  const float* cos;
  const float* sin;
  int64_t tab_stride;
  int tab_rows;
  float* out;            // [B, S, H, D]
  float* lse;            // [B, H, S]
};

__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void bar_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// max / sum over the 16 lanes of each half-warp (both halves hold the same values in the tile loop)
__device__ __forceinline__ float hmax(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float hsum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Writes one finished query row: out[b, s, h, :] and lse[b, h, s].
__device__ __forceinline__ void store_row(const Args& a, int b, int kvh, int r, int d, float acc, float m, float l) {
  int hg = r / a.S, s = r - hg * a.S, h = kvh * a.g + hg;
  bool any = l > 0.0f;  // false only for a call whose position was rejected (device error flag set)
  if (d < a.D) a.out[(((int64_t)b * a.S + s) * a.H + h) * a.D + d] = any ? acc / l : 0.0f;
  if (d == 0) a.lse[((int64_t)b * a.H + h) * a.S + s] = any ? m + logf(l) : -INFINITY;
}

// RotaryEmbedding of element pair (j, j + D/2) of one row (CpuComputeBackend.cs:397-420), as k_rotary_rows rounds it.
__device__ __forceinline__ void rope_pair(float x0, float x1, const float* cr, const float* sr, int j, int half, float& y0,
                                          float& y1) {
  y0 = __fadd_rn(__fmul_rn(x0, cr[j]), __fmul_rn(-x1, sr[j]));
  y1 = __fadd_rn(__fmul_rn(x1, cr[j + half]), __fmul_rn(x0, sr[j + half]));
}

// DC: the head dim when known at compile time (64), else 0 (read from the arguments). ROPE: fused RoPE + append.
template <int R, int DC, bool ROPE>
__global__ void __launch_bounds__(kThreads) k_attn_decode(const Args a) {
  const int D = DC ? DC : a.D;
  extern __shared__ __align__(128) uint8_t smem[];
  const int stages = a.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * kStageBytes);
  uint64_t* empty = full + kStages;
  __shared__ __align__(16) float qs[R][kMaxD];
  __shared__ __align__(16) float ps[kConsumers][R][kTile];
  __shared__ float wm[kConsumers][R], wl[kConsumers][R];
  // the warps' partial outputs, merged after the key loop: they reuse the start of the stage ring (so a 4-stage
  // CTA fits 6 to an SM), written only once every consumer warp is done with its stages
  float (*wacc)[R][kMaxD] = reinterpret_cast<float (*)[R][kMaxD]>(smem);
  __shared__ float cm[R], cl[R];  // this CTA's merged partial, read by cluster rank 0
  __shared__ float ca[R][kMaxD];
  __shared__ volatile int s_abort;
  cg::cluster_group cluster = cg::this_cluster();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = a.rows;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();

  int pos_offset = a.pos_offset, kend = a.L;
  if (a.pos_dev) {
    float pf = a.pos_dev[0];
    pos_offset = (int)pf;
    if (!(pf >= 0.0f) || pos_offset + a.S > a.L || (ROPE && pos_offset + a.S > a.tab_rows)) {
      // outside the cache or the tables: flag it and attend to nothing
      if (split == 0 && threadIdx.x == 0) atomicExch(a.error_flag, 63);
      pos_offset = 0;
      kend = 0;
    }
  }
  if (a.causal) kend = min(kend, pos_offset + a.S);
  // the cluster's CTAs divide the visible keys evenly, in whole tiles
  const int per = ((kend + (int)gridDim.x - 1) / (int)gridDim.x + kTile - 1) / kTile * kTile;
  const int j0 = min(kend, split * per);
  const int j1 = min(kend, j0 + per);
  const int ntiles = (j1 - j0 + kTile - 1) / kTile;
  // new rows sit at positions pos_offset .. pos_offset+S-1, the end of the visible keys: tiles from first_new on hold
  // rows this CTA writes (fused RoPE + append) and are copied only after those writes
  const int first_new = ROPE ? max(0, (pos_offset - j0) / kTile) : ntiles;
  const float* kbase = a.k.p + (int64_t)b * a.k.s0 + (int64_t)kvh * a.k.s1;
  const float* vbase = a.v.p + (int64_t)b * a.v.s0 + (int64_t)kvh * a.v.s1;
  const int half = D >> 1;

  if (warp == kConsumers) {
    // ---------------- producer: tile t -> stage t % stages
    const uint32_t row_bytes = (uint32_t)D * 4;
    int issued = 0;
    for (int t = 0; t < ntiles; t++) {
      if (ROPE && t == first_new) bar_sync(kBarRope, kThreads);
      if (lane == 0 && !s_abort) {
        const int s = t % stages;
        if (t >= stages && !mbar_wait(&empty[s], ((t / stages) & 1) ^ 1)) {
          atomicExch(a.error_flag, 66);
          s_abort = 1;
        } else {
          const int k0 = j0 + t * kTile, nk = min(kTile, j1 - k0);
          uint8_t* st = smem + s * kStageBytes;
          mbar_expect_tx(&full[s], 2u * nk * row_bytes);
          if (a.k.s2 == D) {
            bulk_g2s(st, kbase + (int64_t)k0 * D, nk * row_bytes, &full[s]);
          } else {
            for (int r = 0; r < nk; r++) bulk_g2s(st + r * row_bytes, kbase + (int64_t)(k0 + r) * a.k.s2, row_bytes, &full[s]);
          }
          if (a.v.s2 == D) {
            bulk_g2s(st + kHalfStage, vbase + (int64_t)k0 * D, nk * row_bytes, &full[s]);
          } else {
            for (int r = 0; r < nk; r++)
              bulk_g2s(st + kHalfStage + r * row_bytes, vbase + (int64_t)(k0 + r) * a.v.s2, row_bytes, &full[s]);
          }
          issued = t + 1;
        }
      }
    }
    if (ROPE && first_new >= ntiles) bar_sync(kBarRope, kThreads);  // the consumers always arrive once
    // every copy issued must land before the CTA may exit
    if (lane == 0)
      for (int t = (issued > stages ? issued - stages : 0); t < issued; t++) mbar_wait(&full[t % stages], (t / stages) & 1);
  } else {
    // ---------------- consumers
    constexpr int kCT = 32 * kConsumers;
    if (ROPE) {
      if (kend > 0) {
        // the new key/value rows in this CTA's key range go into the caches (rotated keys) before their tiles load
        for (int t = threadIdx.x; t < a.S * half; t += kCT) {
          int s = t / half, j = t - s * half, pos = pos_offset + s;
          if (pos < j0 || pos >= j1) continue;
          const float* kr = a.kn.p + (int64_t)b * a.kn.s0 + (int64_t)kvh * a.kn.s1 + (int64_t)s * a.kn.s2;
          const float* vr = a.vn.p + (int64_t)b * a.vn.s0 + (int64_t)kvh * a.vn.s1 + (int64_t)s * a.vn.s2;
          float* kd = const_cast<float*>(kbase) + (int64_t)pos * a.k.s2;
          float* vd = const_cast<float*>(vbase) + (int64_t)pos * a.v.s2;
          float y0, y1;
          rope_pair(kr[j], kr[j + half], a.cos + (int64_t)pos * a.tab_stride, a.sin + (int64_t)pos * a.tab_stride, j, half,
                    y0, y1);
          kd[j] = y0;
          kd[j + half] = y1;
          vd[j] = vr[j];
          vd[j + half] = vr[j + half];
        }
      }
      // the writes above are read back by bulk copies (the async proxy)
      asm volatile("fence.proxy.async.global;" ::: "memory");
      bar_arrive(kBarRope, kThreads);
    }
    // query rows of this kv head's group, pre-scaled: row r = (head hg of the group, position s)
    for (int t = threadIdx.x; t < R * kMaxD; t += kCT) {
      int r = t / kMaxD, d = t - r * kMaxD;
      float val = 0.0f;
      if (r < rows && d < a.D) {
        int hg = r / a.S, s = r - hg * a.S, h = kvh * a.g + hg;
        const float* qr = a.q.p + (int64_t)b * a.q.s0 + (int64_t)h * a.q.s1 + (int64_t)s * a.q.s2;
        if (ROPE) {
          int pos = pos_offset + s, j = d < half ? d : d - half;
          float y0, y1;
          rope_pair(qr[j], qr[j + half], a.cos + (int64_t)pos * a.tab_stride, a.sin + (int64_t)pos * a.tab_stride, j, half,
                    y0, y1);
          val = d < half ? y0 : y1;
        } else {
          val = qr[d];
        }
        val = val * a.scale;
      }
      qs[r][d] = val;
    }
    bar_sync(kBarConsumers, kCT);

    const int kk = lane & 15, hf = lane >> 4;  // QKᵀ: this lane's key in the tile and half of the head dims
    const int d0 = 2 * lane;                   // PV: this lane's head-dim pair
    float m[R], l[R], acc0[R], acc1[R];
#pragma unroll
    for (int r = 0; r < R; r++) { m[r] = -INFINITY; l[r] = 0.0f; acc0[r] = 0.0f; acc1[r] = 0.0f; }

    for (int t = warp; t < ntiles; t += kConsumers) {
      const int s = t % stages;
      if (!warp_wait(&full[s], (t / stages) & 1)) {
        if (lane == 0) { atomicExch(a.error_flag, 67); s_abort = 1; }
        break;
      }
      const float* kt = reinterpret_cast<const float*>(smem + s * kStageBytes);
      const float* vt = reinterpret_cast<const float*>(smem + s * kStageBytes + kHalfStage);
      const int k0 = j0 + t * kTile, nk = min(kTile, j1 - k0);
      float sc[R];
#pragma unroll
      for (int r = 0; r < R; r++) sc[r] = 0.0f;
      if (DC == 64) {
        // lane-rotated float4 order: the 8 lanes of each shared-memory phase hit 8 distinct bank groups
        const float4* kr = reinterpret_cast<const float4*>(kt + kk * 64) + hf * 8;
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int d4 = (i + kk) & 7;
          float4 kv = kr[d4];
#pragma unroll
          for (int r = 0; r < R; r++) {
            float4 qv = reinterpret_cast<const float4*>(&qs[r][0])[hf * 8 + d4];
            sc[r] = fmaf(qv.x, kv.x, sc[r]);
            sc[r] = fmaf(qv.y, kv.y, sc[r]);
            sc[r] = fmaf(qv.z, kv.z, sc[r]);
            sc[r] = fmaf(qv.w, kv.w, sc[r]);
          }
        }
      } else {
        const float4* kr = reinterpret_cast<const float4*>(kt + kk * D);
        for (int d4 = hf; d4 < (D >> 2); d4 += 2) {
          float4 kv = kr[d4];
#pragma unroll
          for (int r = 0; r < R; r++) {
            float4 qv = reinterpret_cast<const float4*>(&qs[r][0])[d4];
            sc[r] = fmaf(qv.x, kv.x, sc[r]);
            sc[r] = fmaf(qv.y, kv.y, sc[r]);
            sc[r] = fmaf(qv.z, kv.z, sc[r]);
            sc[r] = fmaf(qv.w, kv.w, sc[r]);
          }
        }
      }
      const int j = k0 + kk;
#pragma unroll
      for (int r = 0; r < R; r++) {
        float sv = sc[r] + __shfl_xor_sync(0xffffffffu, sc[r], 16);
        bool vis = kk < nk && r < rows && (!a.causal || j <= pos_offset + (r % a.S));
        sv = vis ? sv : -INFINITY;
        float mn = fmaxf(m[r], hmax(sv));
        // mn stays -inf only for a row with no visible key so far; it then keeps its zero state
        float alpha = (m[r] == -INFINITY) ? 0.0f : expf(m[r] - mn);
        float p = vis ? expf(sv - mn) : 0.0f;
        float rs = hsum(p);
        l[r] = l[r] * alpha + rs;
        acc0[r] *= alpha;
        acc1[r] *= alpha;
        m[r] = mn;
        if (lane < kTile) ps[warp][r][kk] = p;
      }
      __syncwarp();
#pragma unroll
      for (int j4 = 0; j4 < kTile / 4; j4++) {
        float2 vv[4];
#pragma unroll
        for (int e = 0; e < 4; e++)  // rows past the tile's end hold stale data: read as zero (their p is 0)
          vv[e] = (4 * j4 + e < nk && d0 < D) ? *reinterpret_cast<const float2*>(vt + (4 * j4 + e) * D + d0)
                                              : make_float2(0.f, 0.f);
#pragma unroll
        for (int r = 0; r < R; r++) {
          float4 p4 = reinterpret_cast<const float4*>(&ps[warp][r][0])[j4];
          acc0[r] = fmaf(p4.x, vv[0].x, acc0[r]);
          acc1[r] = fmaf(p4.x, vv[0].y, acc1[r]);
          acc0[r] = fmaf(p4.y, vv[1].x, acc0[r]);
          acc1[r] = fmaf(p4.y, vv[1].y, acc1[r]);
          acc0[r] = fmaf(p4.z, vv[2].x, acc0[r]);
          acc1[r] = fmaf(p4.z, vv[2].y, acc1[r]);
          acc0[r] = fmaf(p4.w, vv[3].x, acc0[r]);
          acc1[r] = fmaf(p4.w, vv[3].y, acc1[r]);
        }
      }
      __syncwarp();  // every lane is done with the stage and with ps
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // merge the warps (fixed order) into this CTA's partial; the partials overwrite stage memory, so every consumer
    // warp first finishes with its stages (every issued copy has landed: each one was awaited by its consumer)
    bar_sync(kBarConsumers, kCT);
#pragma unroll
    for (int r = 0; r < R; r++) {
      if (lane == 0) { wm[warp][r] = m[r]; wl[warp][r] = l[r]; }
      wacc[warp][r][d0] = acc0[r];
      wacc[warp][r][d0 + 1] = acc1[r];
    }
    bar_sync(kBarConsumers, kCT);
    for (int t = threadIdx.x; t < rows * kMaxD; t += kCT) {
      int r = t / kMaxD, d = t - r * kMaxD;
      float M = -INFINITY;
      for (int w = 0; w < kConsumers; w++) M = fmaxf(M, wm[w][r]);
      float L = 0.0f, A = 0.0f;
      if (M != -INFINITY) {
        for (int w = 0; w < kConsumers; w++) {
          float e = wm[w][r] == -INFINITY ? 0.0f : expf(wm[w][r] - M);
          L += wl[w][r] * e;
          A += wacc[w][r][d] * e;
        }
      }
      ca[r][d] = A;
      if (d == 0) { cm[r] = M; cl[r] = L; }
    }
  }
  // rank 0 merges the cluster's partials in rank order; the second barrier keeps every CTA's shared memory alive
  // until rank 0 has read it
  cluster.sync();
  if (cluster.block_rank() == 0) {
    const int n = (int)cluster.num_blocks();
    for (int t = threadIdx.x; t < rows * kMaxD; t += kThreads) {
      int r = t / kMaxD, d = t - r * kMaxD;
      float M = -INFINITY;
      for (int c = 0; c < n; c++) M = fmaxf(M, *cluster.map_shared_rank(&cm[r], c));
      float L = 0.0f, A = 0.0f;
      if (M != -INFINITY) {
        for (int c = 0; c < n; c++) {
          float mc = *cluster.map_shared_rank(&cm[r], c);
          if (mc == -INFINITY) continue;
          float e = expf(mc - M);
          L += *cluster.map_shared_rank(&cl[r], c) * e;
          A += *cluster.map_shared_rank(&ca[r][d], c) * e;
        }
      }
      store_row(a, b, kvh, r, d, A, M, L);
    }
  }
  cluster.sync();
}

// max / sum over a whole warp
__device__ __forceinline__ float wmax32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float wsum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The latency variant for few (batch, kv head) pairs (small decode batches), where each warp gets about one tile and
// the streaming ring cannot pay for itself: no producer warp, every warp loads its own 32-key tile straight from
// global memory (lane j dots key j; V rows prefetched before the QK step), and the kernel may launch early behind the
// previous kernel (programmatic dependent launch). One CTA per (key split, kv head, batch); the splits of one
// (batch, kv head) form a cluster. Each of the 4 warps
// takes 32-key tiles of the CTA's key range; the warps merge in shared memory and cluster rank 0 merges the CTAs'
// partials through distributed shared memory, in rank order.
// DC: the head dim when known at compile time (64), else 0 (read from the arguments). ROPE: fused RoPE + append.
template <int R, int DC, bool ROPE>
__global__ void __launch_bounds__(kDirectThreads) k_attn_decode_direct(const Args a) {
  const int D = DC ? DC : a.D;
  __shared__ __align__(16) float qs[R][kMaxD];
  __shared__ float wm[kDirectWarps][R], wl[kDirectWarps][R];
  __shared__ float wacc[kDirectWarps][R][kMaxD];
  __shared__ float cm[R], cl[R];            // this CTA's merged partial, read by rank 0
  __shared__ float ca[R][kMaxD];
  cg::cluster_group cluster = cg::this_cluster();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = a.rows;
  pdl_trigger();
  pdl_wait();

  int pos_offset = a.pos_offset, kend = a.L;
  if (a.pos_dev) {
    float pf = a.pos_dev[0];
    pos_offset = (int)pf;
    if (!(pf >= 0.0f) || pos_offset + a.S > a.L || (ROPE && pos_offset + a.S > a.tab_rows)) {
      // outside the cache or the tables: flag it and attend to nothing
      if (split == 0 && threadIdx.x == 0) atomicExch(a.error_flag, 63);
      pos_offset = 0;
      kend = 0;
    }
  }
  if (a.causal) kend = min(kend, pos_offset + a.S);
  const int j0 = split * a.keys_per_split;
  const int j1 = min(kend, j0 + a.keys_per_split);
  const float* kbase = a.k.p + (int64_t)b * a.k.s0 + (int64_t)kvh * a.k.s1;
  const float* vbase = a.v.p + (int64_t)b * a.v.s0 + (int64_t)kvh * a.v.s1;
  const int half = D >> 1;

  if (ROPE && kend > 0) {
    // the new key/value rows in this CTA's key range go into the caches first (rotated keys)
    for (int t = threadIdx.x; t < a.S * half; t += kDirectThreads) {
      int s = t / half, j = t - s * half, pos = pos_offset + s;
      if (pos < j0 || pos >= j1) continue;
      const float* kr = a.kn.p + (int64_t)b * a.kn.s0 + (int64_t)kvh * a.kn.s1 + (int64_t)s * a.kn.s2;
      const float* vr = a.vn.p + (int64_t)b * a.vn.s0 + (int64_t)kvh * a.vn.s1 + (int64_t)s * a.vn.s2;
      float* kd = const_cast<float*>(kbase) + (int64_t)pos * a.k.s2;
      float* vd = const_cast<float*>(vbase) + (int64_t)pos * a.v.s2;
      float y0, y1;
      rope_pair(kr[j], kr[j + half], a.cos + (int64_t)pos * a.tab_stride, a.sin + (int64_t)pos * a.tab_stride, j, half, y0, y1);
      kd[j] = y0;
      kd[j + half] = y1;
      vd[j] = vr[j];
      vd[j + half] = vr[j + half];
    }
  }
  // query rows of this kv head's group, pre-scaled: row r = (head hg of the group, position s)
  for (int t = threadIdx.x; t < R * kMaxD; t += kDirectThreads) {
    int r = t / kMaxD, d = t - r * kMaxD;
    float val = 0.0f;
    if (r < rows && d < a.D) {
      int hg = r / a.S, s = r - hg * a.S, h = kvh * a.g + hg;
      const float* qr = a.q.p + (int64_t)b * a.q.s0 + (int64_t)h * a.q.s1 + (int64_t)s * a.q.s2;
      if (ROPE) {
        int pos = pos_offset + s, j = d < half ? d : d - half;
        float y0, y1;
        rope_pair(qr[j], qr[j + half], a.cos + (int64_t)pos * a.tab_stride, a.sin + (int64_t)pos * a.tab_stride, j, half, y0, y1);
        val = d < half ? y0 : y1;
      } else {
        val = qr[d];
      }
      val = val * a.scale;
    }
    qs[r][d] = val;
  }
  __syncthreads();

  const int d0 = 2 * lane;  // this lane's head-dim pair in PV
  float m[R], l[R], acc0[R], acc1[R];
#pragma unroll
  for (int r = 0; r < R; r++) { m[r] = -INFINITY; l[r] = 0.0f; acc0[r] = 0.0f; acc1[r] = 0.0f; }

  for (int t0 = j0 + warp * kDirectTile; t0 < j1; t0 += kDirectWarps * kDirectTile) {
    const int j = t0 + lane;
    const bool in = j < j1;
    const int nk = min(kDirectTile, j1 - t0);
    // this lane's head-dim pair of every V row of the tile, issued first so the loads overlap the QK step
    float2 vv[kDirectTile];
#pragma unroll
    for (int jj = 0; jj < kDirectTile; jj++)
      vv[jj] = (jj < nk && d0 < D) ? *reinterpret_cast<const float2*>(vbase + (int64_t)(t0 + jj) * a.v.s2 + d0)
                                   : make_float2(0.f, 0.f);
    float s[R];
#pragma unroll
    for (int r = 0; r < R; r++) s[r] = 0.0f;
    if (in) {
      const float4* kr = reinterpret_cast<const float4*>(kbase + (int64_t)j * a.k.s2);
#pragma unroll
      for (int d4 = 0; d4 < (DC ? DC / 4 : kMaxD / 4); d4++) {
        if (!DC && d4 >= (D >> 2)) break;
        float4 kv = kr[d4];
#pragma unroll
        for (int r = 0; r < R; r++) {
          float4 qv = *reinterpret_cast<const float4*>(&qs[r][4 * d4]);
          s[r] = fmaf(qv.x, kv.x, s[r]);
          s[r] = fmaf(qv.y, kv.y, s[r]);
          s[r] = fmaf(qv.z, kv.z, s[r]);
          s[r] = fmaf(qv.w, kv.w, s[r]);
        }
      }
    }
    float p[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      bool vis = in && r < rows && (!a.causal || j <= pos_offset + (r % a.S));
      float sv = vis ? s[r] : -INFINITY;
      float mx = wmax32(sv);
      float mn = fmaxf(m[r], mx);
      // mn stays -inf only for a row with no visible key so far; it then keeps its zero state
      float alpha = (m[r] == -INFINITY) ? 0.0f : expf(m[r] - mn);
      p[r] = vis ? expf(sv - mn) : 0.0f;
      float rs = wsum32(p[r]);
      l[r] = l[r] * alpha + rs;
      acc0[r] *= alpha;
      acc1[r] *= alpha;
      m[r] = mn;
    }
    // keys past the tile's end have p = 0 and zero V rows
#pragma unroll
    for (int jj = 0; jj < kDirectTile; jj++) {
#pragma unroll
      for (int r = 0; r < R; r++) {
        float pj = __shfl_sync(0xffffffffu, p[r], jj);
        acc0[r] = fmaf(pj, vv[jj].x, acc0[r]);
        acc1[r] = fmaf(pj, vv[jj].y, acc1[r]);
      }
    }
  }

  // merge the warps (fixed order) into this CTA's partial
#pragma unroll
  for (int r = 0; r < R; r++) {
    if (lane == 0) { wm[warp][r] = m[r]; wl[warp][r] = l[r]; }
    wacc[warp][r][d0] = acc0[r];
    wacc[warp][r][d0 + 1] = acc1[r];
  }
  __syncthreads();
  for (int t = threadIdx.x; t < rows * kMaxD; t += kDirectThreads) {
    int r = t / kMaxD, d = t - r * kMaxD;
    float M = -INFINITY;
    for (int w = 0; w < kDirectWarps; w++) M = fmaxf(M, wm[w][r]);
    float L = 0.0f, A = 0.0f;
    if (M != -INFINITY) {
      for (int w = 0; w < kDirectWarps; w++) {
        float e = wm[w][r] == -INFINITY ? 0.0f : expf(wm[w][r] - M);
        L += wl[w][r] * e;
        A += wacc[w][r][d] * e;
      }
    }
    ca[r][d] = A;
    if (d == 0) { cm[r] = M; cl[r] = L; }
  }
  // rank 0 merges the cluster's partials in rank order; the second barrier keeps every CTA's shared memory alive
  // until rank 0 has read it
  cluster.sync();
  if (cluster.block_rank() == 0) {
    const int n = (int)cluster.num_blocks();
    for (int t = threadIdx.x; t < rows * kMaxD; t += kDirectThreads) {
      int r = t / kMaxD, d = t - r * kMaxD;
      float M = -INFINITY;
      for (int c = 0; c < n; c++) M = fmaxf(M, *cluster.map_shared_rank(&cm[r], c));
      float L = 0.0f, A = 0.0f;
      if (M != -INFINITY) {
        for (int c = 0; c < n; c++) {
          float mc = *cluster.map_shared_rank(&cm[r], c);
          if (mc == -INFINITY) continue;
          float e = expf(mc - M);
          L += *cluster.map_shared_rank(&cl[r], c) * e;
          A += *cluster.map_shared_rank(&ca[r][d], c) * e;
        }
      }
      store_row(a, b, kvh, r, d, A, M, L);
    }
  }
  cluster.sync();
}

}  // namespace dec

template <int R, int DC, bool ROPE>
static cudaError_t launch_decode_r(pai_ctx* ctx, const dec::Args& a, dim3 grid) {
  cudaError_t e = smem_limit(ctx, dec::k_attn_decode<R, DC, ROPE>, (int)dec::smem_bytes(dec::kStages));
  if (e != cudaSuccess) return e;
  // A plain cluster launch: the kernel starts once the previous kernel has finished (its griddepcontrol.wait is then a
  // no-op) but still lets the next kernel launch early. Launched early itself, behind the q/k/v product, it made
  // the decode step slower (batch 1: 1.05 against 0.93 ms per step of the 16-layer model).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(dec::kThreads);
  cfg.dynamicSmemBytes = dec::smem_bytes(a.stages);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeClusterDimension;
  la[0].val.clusterDim.x = (unsigned)a.splits;
  la[0].val.clusterDim.y = 1;
  la[0].val.clusterDim.z = 1;
  cfg.attrs = la;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, dec::k_attn_decode<R, DC, ROPE>, a);
}

// The latency variant is launched early behind the previous kernel (programmatic dependent launch).
template <int R, int DC, bool ROPE>
static cudaError_t launch_direct_r(pai_ctx* ctx, const dec::Args& a, dim3 grid) {
  return launch_pdl_cluster(dec::k_attn_decode_direct<R, DC, ROPE>, grid, dim3(dec::kDirectThreads), 0, ctx->stream,
                            (unsigned)a.splits, a);
}

template <int DC, bool ROPE>
static cudaError_t launch_decode(pai_ctx* ctx, const dec::Args& a, dim3 grid, bool direct) {
  int R = a.rows;
  if (direct) {
    if (R <= 1) return launch_direct_r<1, DC, ROPE>(ctx, a, grid);
    if (R <= 2) return launch_direct_r<2, DC, ROPE>(ctx, a, grid);
    if (R <= 4) return launch_direct_r<4, DC, ROPE>(ctx, a, grid);
    if (R <= 8) return launch_direct_r<8, DC, ROPE>(ctx, a, grid);
    return launch_direct_r<16, DC, ROPE>(ctx, a, grid);
  }
  if (R <= 1) return launch_decode_r<1, DC, ROPE>(ctx, a, grid);
  if (R <= 2) return launch_decode_r<2, DC, ROPE>(ctx, a, grid);
  if (R <= 4) return launch_decode_r<4, DC, ROPE>(ctx, a, grid);
  if (R <= 8) return launch_decode_r<8, DC, ROPE>(ctx, a, grid);
  return launch_decode_r<16, DC, ROPE>(ctx, a, grid);
}

static bool aligned_view(const pai_tensor& t, int vec) {
  if (t.strides[3] != 1) return false;
  if ((uintptr_t)t.base % 16) return false;
  if (t.offset % vec) return false;
  for (int i = 0; i < 3; i++)
    if (t.dims[i] > 1 && t.strides[i] % vec) return false;
  return true;
}

// True when the decode kernel handles this call: at most 16 query rows per kv head, head dim <= 64 (a multiple of
// 4), and K/V views whose rows start on 16-byte boundaries (the bulk copies' alignment).
bool attn_decode_fits(const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, int H, int KVH, int S, int D) {
  int g = H / KVH;
  if (g * S > dec::kMaxRows || D > dec::kMaxD || D % 4) return false;
  return q.strides[3] == 1 && aligned_view(k, 4) && aligned_view(v, 4);
}

// pos_dev: when set, the query position is read on the device and k, v are the whole caches (L = capacity); the
// splits then divide the filled prefix on the device.
// rope: fused RoPE + cache append (q, kn, vn unrotated; a.k / a.v are the caches the new rows are written into).
pai_status attn_decode_run(pai_ctx* ctx, dec::Args& a, bool rope) {
  int kend = (a.causal && !a.pos_dev) ? std::min(a.L, a.pos_offset + a.S) : a.L;
  if (kend < 1) kend = 1;
  a.error_flag = ctx->d_error_flag;
  const int pairs = std::max(1, a.B * a.KVH);
  const bool direct = pairs < dec::kDirectMinPairs;
  if (direct) {
    // latency variant: one 32-key tile per warp (128 keys per CTA) while a cluster of at most 8 CTAs covers the keys,
    // else longer splits
    int kps = dec::kDirectWarps * dec::kDirectTile;
    int need = (kend + dec::kMaxCluster - 1) / dec::kMaxCluster;
    if (need > kps) kps = (need + kps - 1) / kps * kps;
    a.keys_per_split = kps;
    a.splits = (kend + kps - 1) / kps;
  } else {
    // streaming variant. splits: as many as keep the whole grid resident in one wave, at most one cluster of 8, and
    // at most one per 16-key tile. With up to 4 query rows, 3 CTAs per SM fit in shared memory with the 8-stage ring
    // and 6 with a 4-stage ring (32 KB); the consumer warps' QKᵀ / softmax / PV chain is latency-bound, so the
    // shallower ring is taken whenever it lets the grid hold more CTAs (batch 32 x 8 kv heads: 3 splits, 768 CTAs,
    // instead of 1). 8 or 16 query rows: 2 CTAs per SM (registers).
    const int tiles = (kend + dec::kTile - 1) / dec::kTile;
    auto splits_for = [&](int per_sm) {
      return std::max(1, std::min(std::min(dec::kMaxCluster, per_sm * ctx->sm_count / pairs), tiles));
    };
    int stages = dec::kStages;
    a.splits = splits_for(a.rows <= 4 ? 3 : 2);
    if (a.rows <= 4 && splits_for(6) > a.splits) {
      a.splits = splits_for(6);
      stages = dec::kConsumers;
    }
    // ring depth: a multiple of the consumer count, so each stage is always read by the same warp (tile t sits in
    // stage t % stages and is read by warp t % kConsumers) and its barrier phases are awaited in order
    const int max_tiles = ((kend + a.splits - 1) / a.splits + dec::kTile - 1) / dec::kTile;
    a.stages = max_tiles <= dec::kConsumers ? dec::kConsumers : stages;
  }
  dim3 grid((unsigned)a.splits, (unsigned)a.KVH, (unsigned)a.B);
  cudaError_t e;
  if (a.D == 64) e = rope ? launch_decode<64, true>(ctx, a, grid, direct) : launch_decode<64, false>(ctx, a, grid, direct);
  else e = rope ? launch_decode<0, true>(ctx, a, grid, direct) : launch_decode<0, false>(ctx, a, grid, direct);
  PAI_PDL_LAUNCH(e, "attn decode");
  return PAI_OK;
}

static dec::View dview(const pai_tensor& t) {
  return dec::View{static_cast<const float*>(t.base) + t.offset, t.strides[0], t.strides[1], t.strides[2]};
}

pai_status attn_decode_fwd(pai_ctx* ctx, const pai_tensor& q, const pai_tensor& k, const pai_tensor& v, int B, int H,
                           int KVH, int S, int L, int D, float scale, int causal, int pos_offset, float* out, float* lse,
                           const float* pos_dev) {
  dec::Args a{};
  a.pos_dev = pos_dev;
  a.q = dview(q); a.k = dview(k); a.v = dview(v);
  a.B = B; a.H = H; a.KVH = KVH; a.S = S; a.L = L; a.D = D; a.g = H / KVH; a.rows = a.g * S;
  a.pos_offset = pos_offset; a.causal = causal; a.scale = scale;
  a.out = out; a.lse = lse;
  return attn_decode_run(ctx, a, false);
}

}  // namespace pai

// ---------------------------------------------------------------- decode-step entry points (position on the device)
namespace pai {

// k [B, KVH, S, D] (any view) -> cache rows pos .. pos+S-1 of [B, KVH, T, D] (unit head-dim stride).
__global__ void k_kv_append(const float* __restrict__ src, DView sv, float* __restrict__ dst, int64_t d0, int64_t d1,
                            int64_t d2, int KVH, int S, int D, int T, const float* __restrict__ pos, int64_t n,
                            int* error_flag) {
  float pf = pos[0];
  int p = (int)pf;
  if (!(pf >= 0.0f) || p + S > T) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(error_flag, 64);
    return;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    int dd = (int)(r % D); r /= D;
    int s = (int)(r % S); r /= S;
    int h = (int)(r % KVH);
    int b = (int)(r / KVH);
    dst[(int64_t)b * d0 + (int64_t)h * d1 + (int64_t)(p + s) * d2 + dd] = src[dview_offset(sv, i)];
  }
}

// One warp per row of q, k or v [B, heads, S, D] (unit head-dim stride): q rows are rotated into q_out [B, H, S, D],
// k rows rotated into cache positions pos + s, v rows copied there. Rotation as k_rotary_rows (RotaryEmbedding,
// CpuComputeBackend.cs:397-420): y[j] = x[j]·cos[j] − x[j+h]·sin[j], y[j+h] = x[j+h]·cos[j+h] + x[j]·sin[j+h].
struct RopeAppendArgs {
  const float* q; int64_t qs[3];
  const float* k; int64_t ks[3];
  const float* v; int64_t vs[3];
  const float* cos; const float* sin; int64_t tab_stride; int tab_rows;
  float* kc; float* vc; int64_t cs[3];  // caches [B, KVH, T, D]
  float* q_out;
  const float* pos;
  int B, H, KVH, S, D, T;
  int* error_flag;
};

__global__ void k_rope_append(const RopeAppendArgs a) {
  pdl_trigger();
  pdl_wait();
  float pf = a.pos[0];
  int p = (int)pf;
  if (!(pf >= 0.0f) || p + a.S > a.T || p + a.S > a.tab_rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(a.error_flag, 65);
    return;
  }
  const int lane = threadIdx.x & 31, half = a.D >> 1;
  const int64_t nq = (int64_t)a.B * a.H * a.S, nk = (int64_t)a.B * a.KVH * a.S;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t w = warp; w < nq + 2 * nk; w += nwarps) {
    int which = w < nq ? 0 : (w < nq + nk ? 1 : 2);
    int64_t i = which == 0 ? w : (which == 1 ? w - nq : w - nq - nk);
    int heads = which == 0 ? a.H : a.KVH;
    int s = (int)(i % a.S), h = (int)((i / a.S) % heads), b = (int)(i / ((int64_t)a.S * heads));
    const float* src;
    float* dst;
    if (which == 0) {
      src = a.q + b * a.qs[0] + h * a.qs[1] + s * a.qs[2];
      dst = a.q_out + i * a.D;
    } else if (which == 1) {
      src = a.k + b * a.ks[0] + h * a.ks[1] + s * a.ks[2];
      dst = a.kc + b * a.cs[0] + h * a.cs[1] + (int64_t)(p + s) * a.cs[2];
    } else {
      src = a.v + b * a.vs[0] + h * a.vs[1] + s * a.vs[2];
      dst = a.vc + b * a.cs[0] + h * a.cs[1] + (int64_t)(p + s) * a.cs[2];
    }
    if (which == 2) {
      for (int j = lane; j < a.D; j += 32) dst[j] = src[j];
      continue;
    }
    const float* cr = a.cos + (int64_t)(p + s) * a.tab_stride;
    const float* sr = a.sin + (int64_t)(p + s) * a.tab_stride;
    for (int j = lane; j < half; j += 32) {
      float x0 = src[j], x1 = src[j + half];
      dst[j] = __fadd_rn(__fmul_rn(x0, cr[j]), __fmul_rn(-x1, sr[j]));
      dst[j + half] = __fadd_rn(__fmul_rn(x1, cr[j + half]), __fmul_rn(x0, sr[j + half]));
    }
  }
}

static pai_status check_cache(pai_ctx* ctx, const pai_tensor* c, const pai_tensor* x, const char* what) {
  PAI_TRY(check_view(ctx, c, what));
  if (c->rank != 4 || c->dims[0] != x->dims[0] || c->dims[1] != x->dims[1] || c->dims[3] != x->dims[3] ||
      c->strides[3] != 1)
    return set_error(PAI_ERR_ARGUMENT, "%s: cache %s does not fit %s (unit head-dim stride required)", what,
                     shape_str(*c).c_str(), shape_str(*x).c_str());
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_kv_append(pai_ctx* ctx, const pai_tensor* k, const pai_tensor* v, const pai_tensor* k_cache,
                                 const pai_tensor* v_cache, const pai_tensor* pos) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, k, "k"));
  PAI_TRY(check_view(ctx, v, "v"));
  PAI_TRY(check_view(ctx, pos, "pos"));
  if (k->rank != 4 || v->rank != 4 || numel(*pos) != 1)
    return set_error(PAI_ERR_ARGUMENT, "KvAppend: k, v [B, KVH, S, D] and a one-element position expected");
  for (int i = 0; i < 4; i++)
    if (k->dims[i] != v->dims[i]) return set_error(PAI_ERR_ARGUMENT, "KvAppend: k and v shapes differ");
  PAI_TRY(check_cache(ctx, k_cache, k, "k_cache"));
  PAI_TRY(check_cache(ctx, v_cache, v, "v_cache"));
  if (k_cache->dims[2] != v_cache->dims[2] || k->dims[2] > k_cache->dims[2])
    return set_error(PAI_ERR_ARGUMENT, "KvAppend: caches of %d / %d positions for %d new ones", k_cache->dims[2],
                     v_cache->dims[2], k->dims[2]);
  int64_t n = numel(*k);
  if (n == 0) return PAI_OK;
  const pai_tensor* pair[2][2] = {{k, k_cache}, {v, v_cache}};
  for (auto& pr : pair) {
    const pai_tensor* src = pr[0];
    const pai_tensor* dst = pr[1];
    const pai_tensor* sv1[1] = {src};
    DView sv;
    collapse(src->rank, src->dims, sv1, 1, &sv);
    sv.offset = 0;
    k_kv_append<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(fptr(*src), sv, fptr(*dst), dst->strides[0], dst->strides[1],
                                                               dst->strides[2], src->dims[1], src->dims[2], src->dims[3],
                                                               dst->dims[2], fptr(*pos), n, ctx->d_error_flag);
    PAI_LAUNCH_CHECK("kv append");
  }
  return PAI_OK;
}

PAI_API pai_status pai_sdpa_decode(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k_cache, const pai_tensor* v_cache,
                                   const pai_tensor* pos, float scale, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, q, "q"));
  PAI_TRY(check_view(ctx, k_cache, "k_cache"));
  PAI_TRY(check_view(ctx, v_cache, "v_cache"));
  PAI_TRY(check_view(ctx, pos, "pos"));
  if (q->rank != 4 || k_cache->rank != 4 || v_cache->rank != 4 || numel(*pos) != 1)
    return set_error(PAI_ERR_ARGUMENT, "SdpaDecode: q [B,H,S,D], caches [B,KVH,T,D] and a one-element position expected");
  int B = q->dims[0], H = q->dims[1], S = q->dims[2], D = q->dims[3];
  int KVH = k_cache->dims[1], T = k_cache->dims[2];
  for (int i = 0; i < 4; i++)
    if (k_cache->dims[i] != v_cache->dims[i]) return set_error(PAI_ERR_ARGUMENT, "SdpaDecode: k and v caches differ");
  if (k_cache->dims[0] != B || k_cache->dims[3] != D || KVH < 1 || H % KVH)
    return set_error(PAI_ERR_ARGUMENT, "SdpaDecode: q %s does not fit the cache %s", shape_str(*q).c_str(),
                     shape_str(*k_cache).c_str());
  if (!attn_decode_fits(*q, *k_cache, *v_cache, H, KVH, S, D))
    return set_error(PAI_ERR_UNSUPPORTED, "SdpaDecode: needs S*H/KVH <= 16, head dim <= 64 (multiple of 4) and aligned caches");
  int32_t od[4] = {B, S, H, D};
  pai_tensor ro;
  PAI_TRY(alloc_tensor(ctx, 4, od, q->dtype, false, &ro));
  Scratch lse;
  PAI_TRY(scratch(ctx, (size_t)B * H * S * 4, &lse));
  if (numel(ro) > 0) {
    KernelTimerScope timer(ctx, "attn_decode", 8.0 * B * KVH * (double)T * D);
    PAI_TRY(attn_decode_fwd(ctx, *q, *k_cache, *v_cache, B, H, KVH, S, T, D, scale, 1, 0, fptr(ro),
                            static_cast<float*>(lse.p), fptr(*pos)));
  }
  *out = ro;
  return PAI_OK;
}

PAI_API pai_status pai_rope_append(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v,
                                   const pai_tensor* cos_table, const pai_tensor* sin_table, const pai_tensor* k_cache,
                                   const pai_tensor* v_cache, const pai_tensor* pos, pai_tensor* q_out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  const pai_tensor* ins[6] = {q, k, v, cos_table, sin_table, pos};
  const char* names[6] = {"q", "k", "v", "cos", "sin", "pos"};
  for (int i = 0; i < 6; i++) PAI_TRY(check_view(ctx, ins[i], names[i]));
  if (q->rank != 4 || k->rank != 4 || v->rank != 4 || numel(*pos) != 1 || cos_table->rank != 2 || sin_table->rank != 2)
    return set_error(PAI_ERR_ARGUMENT, "RopeAppend: q [B,H,S,D], k and v [B,KVH,S,D], [T,D] tables and a position expected");
  for (int i = 0; i < 4; i++)
    if (k->dims[i] != v->dims[i]) return set_error(PAI_ERR_ARGUMENT, "RopeAppend: k and v shapes differ");
  int B = q->dims[0], H = q->dims[1], S = q->dims[2], D = q->dims[3];
  if (k->dims[0] != B || k->dims[2] != S || k->dims[3] != D || D % 2)
    return set_error(PAI_ERR_ARGUMENT, "RopeAppend: q %s and k %s disagree (or odd head dim)", shape_str(*q).c_str(),
                     shape_str(*k).c_str());
  if (q->strides[3] != 1 || k->strides[3] != 1 || v->strides[3] != 1 || cos_table->strides[1] != 1 ||
      sin_table->strides[1] != 1 || cos_table->strides[0] != sin_table->strides[0])
    return set_error(PAI_ERR_UNSUPPORTED, "RopeAppend: rows must be contiguous and the tables share one layout");
  if (cos_table->dims[1] != D || sin_table->dims[1] != D || sin_table->dims[0] != cos_table->dims[0])
    return set_error(PAI_ERR_ARGUMENT, "RopeAppend: tables must be [T, %d]", D);
  PAI_TRY(check_cache(ctx, k_cache, k, "k_cache"));
  PAI_TRY(check_cache(ctx, v_cache, v, "v_cache"));
  for (int i = 0; i < 3; i++)
    if (k_cache->strides[i] != v_cache->strides[i] || k_cache->dims[i] != v_cache->dims[i])
      return set_error(PAI_ERR_ARGUMENT, "RopeAppend: k and v caches must share one layout");
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, 4, q->dims, q->dtype, false, &r));
  RopeAppendArgs a{};
  a.q = fptr(*q); a.k = fptr(*k); a.v = fptr(*v);
  for (int i = 0; i < 3; i++) { a.qs[i] = q->strides[i]; a.ks[i] = k->strides[i]; a.vs[i] = v->strides[i]; a.cs[i] = k_cache->strides[i]; }
  a.cos = fptr(*cos_table); a.sin = fptr(*sin_table); a.tab_stride = cos_table->strides[0]; a.tab_rows = cos_table->dims[0];
  a.kc = fptr(*k_cache); a.vc = fptr(*v_cache); a.q_out = fptr(r); a.pos = fptr(*pos);
  a.B = B; a.H = H; a.KVH = k->dims[1]; a.S = S; a.D = D; a.T = k_cache->dims[2];
  a.error_flag = ctx->d_error_flag;
  int64_t rows = (int64_t)B * S * (H + 2 * a.KVH);
  if (rows > 0) {
    PAI_PDL_LAUNCH(launch_pdl(k_rope_append, dim3(grid_for(ctx, rows * 32, 256)), dim3(256), 0, ctx->stream, a),
                   "rope append");
  }
  *q_out = r;
  return PAI_OK;
}

PAI_API pai_status pai_attn_decode_step(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v,
                                        const pai_tensor* cos_table, const pai_tensor* sin_table, const pai_tensor* k_cache,
                                        const pai_tensor* v_cache, const pai_tensor* pos, float scale, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  const pai_tensor* ins[6] = {q, k, v, cos_table, sin_table, pos};
  const char* names[6] = {"q", "k", "v", "cos", "sin", "pos"};
  for (int i = 0; i < 6; i++) PAI_TRY(check_view(ctx, ins[i], names[i]));
  if (q->rank != 4 || k->rank != 4 || v->rank != 4 || numel(*pos) != 1 || cos_table->rank != 2 || sin_table->rank != 2)
    return set_error(PAI_ERR_ARGUMENT, "AttnDecodeStep: q [B,H,S,D], k and v [B,KVH,S,D], [T,D] tables and a position expected");
  for (int i = 0; i < 4; i++)
    if (k->dims[i] != v->dims[i]) return set_error(PAI_ERR_ARGUMENT, "AttnDecodeStep: k and v shapes differ");
  int B = q->dims[0], H = q->dims[1], S = q->dims[2], D = q->dims[3], KVH = k->dims[1];
  if (k->dims[0] != B || k->dims[2] != S || k->dims[3] != D || D % 2 || KVH < 1 || H % KVH)
    return set_error(PAI_ERR_ARGUMENT, "AttnDecodeStep: q %s and k %s disagree", shape_str(*q).c_str(), shape_str(*k).c_str());
  if (q->strides[3] != 1 || k->strides[3] != 1 || v->strides[3] != 1 || cos_table->strides[1] != 1 ||
      sin_table->strides[1] != 1 || cos_table->strides[0] != sin_table->strides[0] || cos_table->dims[1] != D ||
      sin_table->dims[1] != D || sin_table->dims[0] != cos_table->dims[0])
    return set_error(PAI_ERR_ARGUMENT, "AttnDecodeStep: rows must be contiguous and the tables [T, %d] of one layout", D);
  PAI_TRY(check_cache(ctx, k_cache, k, "k_cache"));
  PAI_TRY(check_cache(ctx, v_cache, v, "v_cache"));
  for (int i = 0; i < 4; i++)
    if (k_cache->dims[i] != v_cache->dims[i]) return set_error(PAI_ERR_ARGUMENT, "AttnDecodeStep: k and v caches differ");
  if (!attn_decode_fits(*q, *k_cache, *v_cache, H, KVH, S, D))
    return set_error(PAI_ERR_UNSUPPORTED, "AttnDecodeStep: needs S*H/KVH <= 16, head dim <= 64 (multiple of 4) and aligned caches");
  int32_t od[4] = {B, S, H, D};
  pai_tensor ro;
  PAI_TRY(alloc_tensor(ctx, 4, od, q->dtype, false, &ro));
  Scratch lse;
  PAI_TRY(scratch(ctx, (size_t)B * H * S * 4, &lse));
  int T = k_cache->dims[2];
  dec::Args a{};
  a.q = dview(*q); a.k = dview(*k_cache); a.v = dview(*v_cache);
  a.kn = dview(*k); a.vn = dview(*v);
  a.cos = fptr(*cos_table); a.sin = fptr(*sin_table); a.tab_stride = cos_table->strides[0]; a.tab_rows = cos_table->dims[0];
  a.B = B; a.H = H; a.KVH = KVH; a.S = S; a.L = T; a.D = D; a.g = H / KVH; a.rows = a.g * S;
  a.pos_dev = fptr(*pos); a.causal = 1; a.scale = scale;
  a.out = fptr(ro); a.lse = static_cast<float*>(lse.p);
  if (numel(ro) > 0) {
    KernelTimerScope timer(ctx, "attn_decode", 8.0 * B * KVH * (double)T * D);
    PAI_TRY(attn_decode_run(ctx, a, true));
  }
  *out = ro;
  return PAI_OK;
}
