// LSE merge of many partials of a row, spread over the warps of a CTA.
//
// A long request decoded with many KV splits (or one slice of a sequence-split request) leaves
// few rows (batch x heads) and many partials per row.  A grid of one CTA per row (or per few
// rows) then holds a handful of SMs, each streaming every partial of its rows one batch of
// loads after another.  Here a CTA takes one 128-column chunk of a row and its warps take the
// partials in turn, so the loads of all partials are in flight at once across D / 128 CTAs per
// row.  The merge is the split-KV merge of packed_mla_decode_gf_fwd
// (deployment/patches/rolaq_sglang.patch:98-111): weights exp(lse_k - max), the weighted sum
// of the normalised partials divided by the sum of the weights, lse = max + log(sum).
#pragma once

#include "common.cuh"

namespace rolaq {
namespace wide {

constexpr int kWarps = 8;                 // warps of a CTA
constexpr int kThreads = kWarps * 32;
constexpr int kCols = 128;                // columns of a row per CTA: a float4 per lane
constexpr int kMinParts = 16;             // fewer partials: the per-row kernels are as fast

__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Chunk [c0, c0 + 128) of one row merged over n partials: partial k's values at
// o + k * part_stride (column 0 first), its lse at lse[k * lse_stride].  Warp w takes
// partials w, w + 8, w + 16, .., eight loads in flight before any is used; lane l holds
// columns c0 + 4l .. c0 + 4l + 3, and columns at or past d are neither read nor returned
// (d and c0 multiples of 4, rows 16-byte aligned).  Empty partials (lse = -inf) are masked,
// never multiplied.  The warps' sums meet in `red` and are added in warp order, so the result
// does not depend on scheduling.  Every thread of the CTA must call it (it synchronises the
// CTA once); warp 0 receives the merged values in `res` and the return value is the merged
// lse there (-inf for a row with no tokens, whose values are 0).
__device__ __forceinline__ float merge_chunk(const float* __restrict__ o, int64_t part_stride,
                                             const float* __restrict__ lse, int64_t lse_stride, int n, int c0,
                                             int d, float4 (*red)[32], float4& res) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m = -INFINITY;
  for (int k = lane; k < n; k += 32) m = fmaxf(m, lse[k * lse_stride]);
  m = wmax(m);
  const float mref = m == -INFINITY ? 0.f : m;
  const int col = c0 + 4 * lane;
  const bool live = col < d;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const int mine = warp < n ? (n - warp + kWarps - 1) / kWarps : 0;  // this warp's partials
  for (int i0 = 0; i0 < mine; i0 += 32) {
    const int cnt = min(32, mine - i0);
    const float lv = lane < cnt ? lse[int64_t(warp + kWarps * (i0 + lane)) * lse_stride] : -INFINITY;
    const float wl = lv != -INFINITY ? __expf(lv - mref) : 0.f;  // weight of partial i0 + lane
    for (int q = 0; q < cnt; q += 8) {
      float4 v[8];
      float w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        w[u] = __shfl_sync(0xFFFFFFFFu, wl, (q + u) & 31);
        if (q + u >= cnt) w[u] = 0.f;
        const int64_t k = warp + kWarps * (i0 + min(q + u, cnt - 1));
        v[u] = live ? *reinterpret_cast<const float4*>(o + k * part_stride + col) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc.x = w[u] > 0.f ? fmaf(w[u], v[u].x, acc.x) : acc.x;
        acc.y = w[u] > 0.f ? fmaf(w[u], v[u].y, acc.y) : acc.y;
        acc.z = w[u] > 0.f ? fmaf(w[u], v[u].z, acc.z) : acc.z;
        acc.w = w[u] > 0.f ? fmaf(w[u], v[u].w, acc.w) : acc.w;
      }
    }
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp != 0) return -INFINITY;
  float den = 0.f;
  for (int k = lane; k < n; k += 32) {
    const float lv = lse[k * lse_stride];
    den += lv != -INFINITY ? __expf(lv - mref) : 0.f;
  }
  den = wsum(den);
  float4 s = red[0][lane];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) {
    const float4 t = red[w][lane];
    s.x += t.x;
    s.y += t.y;
    s.z += t.z;
    s.w += t.w;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  res = make_float4(s.x * inv, s.y * inv, s.z * inv, s.w * inv);
  return den > 0.f ? mref + logf(den) : -INFINITY;
}

__device__ __forceinline__ uint2 to_bf16x4(float4 v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

}  // namespace wide
}  // namespace rolaq
