// Per-sequence position / padding update after a commit, shared by the
// stand-alone position update and the fused commit-round kernel.
//
// For sequence b and accepted columns j < width (helper/opd_generate.py:556-558,
// 644-650 of the reference):
//   pad_rows[owners[b]][past + j] = newly_padded[b][j]
//   pad_live[b][past + j]         = newly_padded[b][j]
//   positions[b][j]               = past_positions[b] + #unpadded columns <= j
//   past_positions[b]             = positions[b][width - 1]
#pragma once
#include "common.cuh"

namespace speckv {

struct PositionArgs {
  uint8_t* pad_rows;        // (pad_count, prs) or null
  long long prs, pad_count;
  const int64_t* owners;    // (batch,) row of pad_rows owned by sequence b
  uint8_t* pad_live;        // (batch, pls) or null
  long long pls;
  const uint8_t* np;        // newly padded (batch, npsb), unit column stride
  long long npsb;
  int64_t* positions;       // (batch, psb)
  long long psb;
  int64_t* past_positions;  // (batch,)
};

// One warp updates sequence b; every lane of the warp must call it.
__device__ __forceinline__ void position_row(const PositionArgs& a, long long b, long long past, long long width,
                                             int lane, unsigned long long* err) {
  long long owner = -1;
  if (a.pad_rows != nullptr) {
    owner = a.owners[b];
    if (owner < 0 || owner >= a.pad_count) {
      if (lane == 0) record_error(err, SPECKV_DERR_OWNER_INDEX, owner);
      owner = -1;
    }
  }
  long long carry = a.past_positions[b];
  for (long long j0 = 0; j0 < width; j0 += 32) {
    const long long j = j0 + lane;
    const bool in = j < width;
    const uint8_t padded = in ? a.np[b * a.npsb + j] : 1;
    if (in) {
      if (owner >= 0) a.pad_rows[owner * a.prs + past + j] = padded;
      if (a.pad_live != nullptr) a.pad_live[b * a.pls + past + j] = padded;
    }
    int inc = (in && !padded) ? 1 : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (in) a.positions[b * a.psb + j] = carry + inc;
    carry += __shfl_sync(0xffffffffu, inc, 31);
  }
  if (lane == 0) a.past_positions[b] = carry;
}

}  // namespace speckv
