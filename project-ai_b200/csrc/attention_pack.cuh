// Attention operand packing, shared by the tensor-core forward (attention_tc.cu, which holds the kernel) and
// backward (attention_tc_bwd.cu).
#pragma once

#include "common.cuh"

namespace pai {

// One operand view [B, X, R, D] (X heads, R positions) to pack into tf32 hi/lo SWIZZLE_128B tiles of `blk` positions.
struct AttnPackArgs {
  const float* src;
  int64_t s_b, s_x, s_r, s_d;  // element strides of the [B, X, R, D] view
  int X, R, D;
  int blk;        // sequence positions per packed tile (128 for Q, 64 for K/V)
  int transpose;  // 0: tile rows = positions, cols = d;  1: tile rows = d, cols = positions
  float scale;
  int nblk;       // tiles along R
  float* out;     // [B·X][nblk] tiles: [hi kb0][hi kb1][lo kb0][lo kb1], kb = 32 columns
};

constexpr int kAttnPackMax = 8;  // operands one launch packs

// Packs n (1..kAttnPackMax) operands of a B-batch attention call with one launch (operand i: nblk·B·X tiles).
pai_status attn_pack_launch(pai_ctx* ctx, const AttnPackArgs* packs, int n, int B);

}  // namespace pai
