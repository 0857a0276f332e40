// Absorbed MLA decode attention over the packed INT2 cache, sm_100a.
//
// Reference behaviour: the upstream packed_mla_decode_gf_fwd called at
// deployment/patches/rolaq_sglang.patch:51-111 (split-KV online softmax over INT2
// latents, one extra split over the BF16 window rows, LSE merge), with queries in
// the rotated frame (deployment/sglang/srt/mem_cache/rolaq_mla.py:56-71).
//
// Grid (num_splits + 1, batch).  A CTA of 4 warps streams the 64-token pages of its
// split: TMA copies a page's codes and k_pe (128-byte or 64-byte swizzled) and a bulk
// copy its (scale, zero) params into a 3-stage mbarrier pipeline.  The INT2 codes are
// never dequantised to a tensor: with c_hat = (c - zero) * scale per 128-group,
//   q . c_hat     = sum_g scale_g * (q_g . c - zero_g * sum(q_g))
//   sum_t p_t c_hat_t = sum_t (p_t * scale_g,t) * c_t - sum_t p_t * scale_g,t * zero_g,t
// so both contractions run on the tensor cores with the raw codes as BF16 operands.
// A code c becomes the BF16 value 128 + c (or 128 + 4c) with one AND/OR: bits
// 0x4300 | c are exactly 128 + c; the 128 (and the 1/4 on the matching query
// elements) are removed algebraically.
//   QK^T : S[tok, head] = codes[tok, :] x q^T          (m16n8k16, M = 16 tokens)
//   PV   : O^T[elem, head] += codes^T[elem, tok] x P'  (m16n8k16, M = 16 elements)
// The window split reads the BF16 ring rows (or the INT2 codes when a ring row no
// longer belongs to the slot) in FP32 on the CUDA cores.
#include "kernels.cuh"
#include "merge.cuh"

namespace rolaq {

constexpr uint32_t kMagic = 0x43004300u;    // BF16x2 {128, 128}: QK codes, 128 + c
constexpr uint32_t kMagic16 = 0x64006400u;  // FP16x2 {1024, 1024}: PV codes, 1024 + c

__device__ __forceinline__ uint32_t hsub_magic16(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  h = __hsub2(h, __half2half2(__ushort_as_half(0x6400)));
  return *reinterpret_cast<uint32_t*>(&h);
}
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kPage = 64;
constexpr int kDecodeThreads = 128;
constexpr int kMaxWindow = 32;

template <int D, int DR, int H>
struct DecodeCfg {
  static constexpr int NG = D / 128;
  static constexpr int HN = H / 8;
  static constexpr int CODE_ROW = D / 4;  // bytes of codes per token
  static constexpr int KS_CODE = D / 16;
  static constexpr int KS_PE = DR / 16;
  static constexpr int QROW = D + DR + 8;  // BF16 per query row in smem (bank padding)
  static constexpr int MT = D / 64;        // PV m-tiles (16 elements) per warp
  static constexpr int PSTRIDE = (HN % 2 == 1) ? H : H + 8;  // odd number of 16-byte chunks
  static constexpr int ST_CODES = kPage * CODE_ROW;
  static constexpr int ST_ROPE = kPage * DR * 2;
  static constexpr int ST_PARAMS = kPage * NG * 8;
  static constexpr int ST_BYTES = ((ST_CODES + ST_ROPE + ST_PARAMS + 1023) / 1024) * 1024;
  static constexpr int STAGES = 3;
  static constexpr int Q_BYTES = H * QROW * 2;
  static constexpr int P_BYTES = 2 * NG * kPage * PSTRIDE * 2;
  static constexpr int F_FLOATS = 2 * NG * H + 2 * 4 * H + 4 * NG * H;
  static constexpr size_t PIPE_SMEM = size_t(STAGES) * ST_BYTES + Q_BYTES + P_BYTES + F_FLOATS * 4 + 64;
  static constexpr size_t WIN_SMEM = size_t(kMaxWindow) * (D + DR) * 4 + size_t(kMaxWindow) * H * 4;
  static constexpr size_t SMEM = (PIPE_SMEM > WIN_SMEM ? PIPE_SMEM : WIN_SMEM) + 1024;
  static_assert(D == 256 || D == 512, "latent width");
  static_assert(H % 8 == 0, "heads");
};

// Byte offset of (row, byte) inside a TMA tile whose rows are `row_bytes` long and
// swizzled with the matching CU_TENSOR_MAP_SWIZZLE mode (128 B or 64 B rows).
template <int RB>
__device__ __forceinline__ uint32_t swz(int row, int byte) {
  const int chunk = byte >> 4;
  const int phys = RB == 128 ? (chunk ^ (row & 7)) : (chunk ^ ((row >> 1) & 3));
  return static_cast<uint32_t>(row * RB + (phys << 4) + (byte & 15));
}

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

template <int D, int DR, int H>
__device__ void window_split(const DecodeArgs& a, uint8_t* smem, int b, int L) {
  using C = DecodeCfg<D, DR, H>;
  const int tid = threadIdx.x;
  const int P = a.cache.sink, W = a.cache.recent;
  const int lo = min(P, L);
  const int hs = max(lo, L - W);
  int rs = 0, re = L;
  if (a.token_range != nullptr) {
    rs = max(0, a.token_range[2 * b]);
    re = min(L, a.token_range[2 * b + 1]);
  }
  // window positions [0, lo) u [hs, L), restricted to [rs, re)
  const int s1 = min(max(rs, 0), lo), e1 = max(min(re, lo), s1);
  const int s2 = min(max(rs, hs), L), e2 = max(min(re, L), s2);
  const int n1 = e1 - s1;
  const int nw = n1 + (e2 - s2);
  float* kw = reinterpret_cast<float*>(smem);  // [nw][D + DR]
  float* pr = kw + kMaxWindow * (D + DR);      // [H][nw]
  __shared__ float wm[H], wl[H];
  for (int idx = tid; idx < nw * (D + DR); idx += blockDim.x) {
    const int p = idx / (D + DR);
    const int e = idx % (D + DR);
    const int pos = p < n1 ? s1 + p : s2 + (p - n1);
    const int64_t page = a.page_table[b * a.pt_stride + pos / kPage];
    float v = 0.f;
    if (page >= 0 && (page + 1) * kPage <= a.cache.num_slots) {
      const int64_t slot = page * kPage + pos % kPage;
      if (e < D) {
        int64_t r = a.cache.rows ? a.cache.rows[slot] : -1;
        const bool owned = r >= 0 && r < a.cache.num_ring_rows && a.cache.owners[r] == slot;
        if (owned) {
          v = bf16f(a.cache.hp[r * D + e]);
        } else {
          const uint32_t c = (a.cache.codes[slot * (D / 4) + e / 4] >> (2 * (e % 4))) & 3u;
          const float2 sz = reinterpret_cast<const float2*>(a.cache.params)[slot * (D / 128) + e / 128];
          v = __fmul_rn(__fsub_rn(static_cast<float>(c), sz.y), sz.x);
        }
      } else {
        v = bf16f(a.cache.rope[slot * DR + (e - D)]);
      }
    } else if (e == 0) {
      report(a.err, ROLAQ_DEV_BAD_PAGE);
    }
    kw[idx] = v;
  }
  __syncthreads();
  const uint16_t* qb = a.q + b * a.q_sb;
  for (int u = tid; u < H * nw; u += blockDim.x) {
    const int h = u / nw, p = u % nw;
    const uint16_t* qh = qb + h * a.q_sh;
    const float* k = kw + p * (D + DR);
    const int pos = p < n1 ? s1 + p : s2 + (p - n1);
    const int64_t page = a.page_table[b * a.pt_stride + pos / kPage];
    float s = 0.f;
    for (int e = 0; e < D + DR; ++e) s = fmaf(bf16f(qh[e]), k[e], s);
    // a row whose page is out of range takes no weight (the INT2 splits skip such tokens too)
    pr[h * nw + p] = (page >= 0 && (page + 1) * kPage <= a.cache.num_slots) ? s * a.sm_scale : -INFINITY;
  }
  __syncthreads();
  if (tid < H) {
    float m = -INFINITY;
    for (int p = 0; p < nw; ++p) m = fmaxf(m, pr[tid * nw + p]);
    float l = 0.f;
    for (int p = 0; p < nw; ++p) {
      const float x = pr[tid * nw + p];
      const float e = x != -INFINITY ? __expf(x - m) : 0.f;
      pr[tid * nw + p] = e;
      l += e;
    }
    wm[tid] = m;
    wl[tid] = l;
  }
  __syncthreads();
  const int S = a.num_splits + 1;
  for (int u = tid; u < H * D; u += blockDim.x) {
    const int h = u / D, j = u % D;
    float o = 0.f;
    for (int p = 0; p < nw; ++p) o = fmaf(pr[h * nw + p], kw[p * (D + DR) + j], o);
    const int64_t row = (static_cast<int64_t>(b) * H + h) * S + a.num_splits;
    a.part_o[row * D + j] = wl[h] > 0.f ? o / wl[h] : 0.f;
  }
  if (tid < H) {
    const int64_t row = (static_cast<int64_t>(b) * H + tid) * S + a.num_splits;
    a.part_lse[row] = wl[tid] > 0.f ? wm[tid] + logf(wl[tid]) : -INFINITY;
  }
}

// The window split on its own (used with the tcgen05 INT2 kernel): grid = (batch, H / 4),
// four heads per CTA, one warp per head.  Same arithmetic as window_split (the q.k dot
// product runs as four interleaved partial sums); the rows are gathered once per row
// (lookups by one thread, elements by a warp, coalesced) into shared rows padded to an odd
// stride, so that a lane per row reads them without bank conflicts.
constexpr int kWinHeads = 4;
template <int D, int DR>
constexpr size_t window_rows_smem() {
  return (size_t(kMaxWindow) * (D + DR + 1) + size_t(kWinHeads) * (D + DR) + size_t(kWinHeads) * kMaxWindow) * 4;
}

template <int D, int DR, int H>
__global__ void __launch_bounds__(kWinHeads * 32) window_rows_kernel(const DecodeArgs a) {
  constexpr int KW = D + DR, KP = KW + 1;
  extern __shared__ float wsm[];
  float* kw = wsm;                        // [kMaxWindow][KP]
  float* qf = kw + kMaxWindow * KP;       // [kWinHeads][KW]
  float* pr = qf + kWinHeads * KW;        // [kWinHeads][kMaxWindow]
  __shared__ float wm[kWinHeads], wl[kWinHeads];
  __shared__ int64_t rslot[kMaxWindow];
  __shared__ int64_t rrow[kMaxWindow];
  const int b = blockIdx.x, h0 = blockIdx.y * kWinHeads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int L = a.seq_lens[b];
  if (L < 0) L = 0;
  if (L > a.max_pages * kPage) L = a.max_pages * kPage;
  const int P = a.cache.sink, W = a.cache.recent;
  const int lo = min(P, L);
  const int hs = max(lo, L - W);
  int rs = 0, re = L;
  if (a.token_range != nullptr) {
    rs = max(0, a.token_range[2 * b]);
    re = min(L, a.token_range[2 * b + 1]);
  }
  const int s1 = min(max(rs, 0), lo), e1 = max(min(re, lo), s1);
  const int s2 = min(max(rs, hs), L), e2 = max(min(re, L), s2);
  const int n1 = e1 - s1;
  const int nw = n1 + (e2 - s2);  // <= sink + recent <= kMaxWindow (checked by the host)
  if (tid < nw) {  // per row: slot and the ring row that holds it (if any); first, as the longest chain
    const int pos = tid < n1 ? s1 + tid : s2 + (tid - n1);
    const int64_t page = a.page_table[b * a.pt_stride + pos / kPage];
    int64_t slot = -1, r = -1;
    if (page >= 0 && (page + 1) * kPage <= a.cache.num_slots) {
      slot = page * kPage + pos % kPage;
      r = a.cache.rows ? a.cache.rows[slot] : -1;
      if (!(r >= 0 && r < a.cache.num_ring_rows && a.cache.owners[r] == slot)) r = -1;
    } else {
      report(a.err, ROLAQ_DEV_BAD_PAGE);
    }
    rslot[tid] = slot;
    rrow[tid] = r;
  }
  // queries of the 4 heads as FP32, 8 BF16 per 16-byte load (rows 16-byte aligned on this path)
  for (int idx = tid; idx < kWinHeads * (KW / 8); idx += blockDim.x) {
    const int h = idx / (KW / 8), c = idx % (KW / 8);
    const uint4 w = *reinterpret_cast<const uint4*>(a.q + b * a.q_sb + (h0 + h) * a.q_sh + 8 * c);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      qf[h * KW + 8 * c + 2 * u] = __uint_as_float(ws[u] << 16);
      qf[h * KW + 8 * c + 2 * u + 1] = __uint_as_float(ws[u] & 0xFFFF0000u);
    }
  }
  __syncthreads();
  static_assert(D % 256 == 0 && DR % 8 == 0 && DR / 8 <= 32, "window row gather shape");
  for (int p = warp; p < nw; p += kWinHeads) {  // warp per row, 16-byte loads
    const int64_t slot = rslot[p], r = rrow[p];
    float* dst = kw + p * KP;
    if (slot < 0) {
      for (int e = lane; e < KW; e += 32) dst[e] = 0.f;
      continue;
    }
    if (r >= 0) {
#pragma unroll
      for (int u = 0; u < D / 256; ++u) {
        const int e0 = 8 * lane + 256 * u;
        const uint4 w = *reinterpret_cast<const uint4*>(a.cache.hp + r * D + e0);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          dst[e0 + 2 * v] = __uint_as_float(ws[v] << 16);
          dst[e0 + 2 * v + 1] = __uint_as_float(ws[v] & 0xFFFF0000u);
        }
      }
    } else {
      for (int e0 = 16 * lane; e0 < D; e0 += 16 * 32) {  // 16 codes (one 32-bit word) per step
        const uint32_t cw = *reinterpret_cast<const uint32_t*>(a.cache.codes + slot * (D / 4) + e0 / 4);
        const float2 sz = reinterpret_cast<const float2*>(a.cache.params)[slot * (D / 128) + e0 / 128];
#pragma unroll
        for (int v = 0; v < 16; ++v)
          dst[e0 + v] = __fmul_rn(__fsub_rn(static_cast<float>((cw >> (2 * v)) & 3u), sz.y), sz.x);
      }
    }
    if (lane < DR / 8) {
      const uint4 w = *reinterpret_cast<const uint4*>(a.cache.rope + slot * DR + 8 * lane);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        dst[D + 8 * lane + 2 * v] = __uint_as_float(ws[v] << 16);
        dst[D + 8 * lane + 2 * v + 1] = __uint_as_float(ws[v] & 0xFFFF0000u);
      }
    }
  }
  __syncthreads();
  {  // warp = head, lane = row
    const int h = warp;
    float sc = -INFINITY;
    if (lane < nw && rslot[lane] >= 0) {  // four interleaved partial sums (KW is a multiple of 4);
                                          // a row whose page is out of range takes no weight
      const float* k = kw + lane * KP;
      const float* qh = qf + h * KW;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
      for (int e = 0; e < KW; e += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u] = fmaf(qh[e + u], k[e + u], acc[u]);
      }
      sc = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * a.sm_scale;
    }
    float m = sc;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    const float ex = sc != -INFINITY ? __expf(sc - m) : 0.f;
    pr[h * kMaxWindow + lane] = ex;
    __syncwarp();
    if (lane == 0) {  // the sum in row order, as window_split
      float l = 0.f;
      for (int p = 0; p < nw; ++p) l += pr[h * kMaxWindow + p];
      wm[h] = m;
      wl[h] = l;
    }
  }
  __syncthreads();
  const int S = a.num_splits + 1;
  static_assert(D % (kWinHeads * 32) == 0, "latent elements per thread");
  constexpr int JT = D / (kWinHeads * 32);  // elements per thread, for all kWinHeads heads
  float o[kWinHeads][JT];
#pragma unroll
  for (int h = 0; h < kWinHeads; ++h)
#pragma unroll
    for (int c = 0; c < JT; ++c) o[h][c] = 0.f;
  for (int p = 0; p < nw; ++p) {
    float kv[JT];
#pragma unroll
    for (int c = 0; c < JT; ++c) kv[c] = kw[p * KP + tid + c * kWinHeads * 32];
#pragma unroll
    for (int h = 0; h < kWinHeads; ++h) {
      const float w = pr[h * kMaxWindow + p];
#pragma unroll
      for (int c = 0; c < JT; ++c) o[h][c] = fmaf(w, kv[c], o[h][c]);
    }
  }
#pragma unroll
  for (int h = 0; h < kWinHeads; ++h) {
    const int64_t row = (static_cast<int64_t>(b) * H + h0 + h) * S + a.num_splits;
#pragma unroll
    for (int c = 0; c < JT; ++c)
      a.part_o[row * D + tid + c * kWinHeads * 32] = wl[h] > 0.f ? o[h][c] / wl[h] : 0.f;
  }
  if (tid < kWinHeads) {
    const int64_t row = (static_cast<int64_t>(b) * H + h0 + tid) * S + a.num_splits;
    a.part_lse[row] = wl[tid] > 0.f ? wm[tid] + logf(wl[tid]) : -INFINITY;
  }
}

template <int D, int DR, int H>
__global__ void __launch_bounds__(kDecodeThreads, 2)
    decode_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_rope,
                  const DecodeArgs a) {
  using C = DecodeCfg<D, DR, H>;
  constexpr int NG = C::NG, HN = C::HN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint16_t* qk = reinterpret_cast<uint16_t*>(smem + C::STAGES * C::ST_BYTES);
  uint16_t* pbuf = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(qk) + C::Q_BYTES);
  float* corr = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(pbuf) + C::P_BYTES);  // [NG][H]
  float* qsum = corr + NG * H;                                                             // [NG][H]
  float* red = qsum + NG * H;                                                              // [2][4][H]
  float* yred = red + 2 * 4 * H;                                                           // [4][NG][H]
  uint64_t* full = reinterpret_cast<uint64_t*>(yred + 4 * NG * H);
  int* bad = reinterpret_cast<int*>(full + C::STAGES);

  const int b = blockIdx.y;
  const int split = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, qi = lane & 3;
  const int S = a.num_splits + 1;
  int L = a.seq_lens[b];
  if (L < 0) L = 0;
  if (L > a.max_pages * kPage) {
    if (tid == 0) report(a.err, ROLAQ_DEV_BAD_REQ);
    L = a.max_pages * kPage;
  }
  if (split == a.num_splits) {
    window_split<D, DR, H>(a, smem, b, L);
    return;
  }

  const int P = a.cache.sink, W = a.cache.recent;
  int lo = min(P, L);
  int hi = max(lo, L - W);
  if (a.token_range != nullptr) {
    lo = max(lo, a.token_range[2 * b]);
    hi = max(lo, min(hi, a.token_range[2 * b + 1]));
  }
  const int first_page = lo / kPage;
  const int npages = hi > lo ? (hi - 1) / kPage - first_page + 1 : 0;
  const int pps = (npages + a.num_splits - 1) / a.num_splits;
  const int p0 = first_page + split * pps;
  const int p1 = min(first_page + npages, p0 + pps);
  if (p0 >= p1) {
    for (int u = tid; u < H * D; u += blockDim.x) {
      const int h = u / D, j = u % D;
      a.part_o[((static_cast<int64_t>(b) * H + h) * S + split) * D + j] = 0.f;
    }
    if (tid < H) a.part_lse[(static_cast<int64_t>(b) * H + tid) * S + split] = -INFINITY;
    return;
  }

  // ---- pipeline set-up --------------------------------------------------------------
  auto issue = [&](int page_idx, int stage) {
    uint8_t* st = smem + stage * C::ST_BYTES;
    const int64_t page = a.page_table[b * a.pt_stride + page_idx];
    if (page < 0 || (page + 1) * kPage > a.cache.num_slots) {
      bad[stage] = 1;
      report(a.err, ROLAQ_DEV_BAD_PAGE);
      mbar_arrive(&full[stage]);
      return;
    }
    bad[stage] = 0;
    mbar_expect_tx(&full[stage], C::ST_CODES + C::ST_ROPE + C::ST_PARAMS);
    tma_load_2d(st, &tm_codes, &full[stage], 0, static_cast<int32_t>(page * kPage));
    tma_load_2d(st + C::ST_CODES, &tm_rope, &full[stage], 0, static_cast<int32_t>(page * kPage));
    bulk_load(st + C::ST_CODES + C::ST_ROPE, a.cache.params + page * kPage * NG * 2, C::ST_PARAMS, &full[stage]);
  };
  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    prefetch_tensormap(&tm_codes);
    prefetch_tensormap(&tm_rope);
    for (int s = 0; s < 2 && p0 + s < p1; ++s) issue(p0 + s, s);
  }

  // ---- queries: permuted / scaled copy for the MMA B operand, correction sums ---------
  // Within each 16-element block the MMA k index kk maps to latent element
  // e(kk): 2i -> 2i, 2i+1 -> 2i+8, 2i+8 -> 2i+1, 2i+9 -> 2i+9 (i = 0..3), matching the
  // register layout of the expanded codes; odd elements carry the factor 1/4.
  const uint16_t* qb = a.q + b * a.q_sb;
  for (int idx = tid; idx < H * (D + DR); idx += blockDim.x) {
    const int h = idx / (D + DR), e = idx % (D + DR);
    const uint16_t v = qb[h * a.q_sh + e];
    if (e < D) {
      const int w = e & 15;
      const int kk = (w & 1) ? (w < 8 ? w + 7 : w) : (w < 8 ? w : w - 7);
      uint16_t out = v;
      if (w & 1) {
        const float f = bf16f(v) * 0.25f;
        out = static_cast<uint16_t>(__float_as_uint(f) >> 16);  // exact: power-of-two scale
      }
      qk[h * C::QROW + (e & ~15) + kk] = out;
    } else {
      qk[h * C::QROW + e] = v;
    }
  }
  for (int u = tid; u < H * NG; u += blockDim.x) {
    const int h = u / NG, gr = u % NG;
    float s = 0.f, c = 0.f;
    for (int e = gr * 128; e < gr * 128 + 128; ++e) {
      const float v = bf16f(qb[h * a.q_sh + e]);
      s += v;
      c = fmaf(v, (e & 1) ? 32.f : 128.f, c);
    }
    qsum[gr * H + h] = s;
    corr[gr * H + h] = c;
  }
  __syncthreads();

  // per-lane constants for the heads this lane owns: 8t + 2*qi + cc
  float lcorr[NG][HN][2], lqsum[NG][HN][2];
#pragma unroll
  for (int gr = 0; gr < NG; ++gr)
#pragma unroll
    for (int t = 0; t < HN; ++t)
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        lcorr[gr][t][cc] = corr[gr * H + 8 * t + 2 * qi + cc];
        lqsum[gr][t][cc] = qsum[gr * H + 8 * t + 2 * qi + cc];
      }

  float m_run[HN][2], l_part[HN][2], y_part[NG][HN][2];
#pragma unroll
  for (int t = 0; t < HN; ++t)
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      m_run[t][cc] = -INFINITY;
      l_part[t][cc] = 0.f;
#pragma unroll
      for (int gr = 0; gr < NG; ++gr) y_part[gr][t][cc] = 0.f;
    }
  float o[C::MT][HN][4];
#pragma unroll
  for (int mt = 0; mt < C::MT; ++mt)
#pragma unroll
    for (int t = 0; t < HN; ++t)
#pragma unroll
      for (int k = 0; k < 4; ++k) o[mt][t][k] = 0.f;

  const float sl2 = a.sm_scale * kLog2e;
  const int e0 = warp * (D / 4);  // first latent element of this warp's PV slice
  const int grw = e0 / 128;       // its quantisation group
  const uint32_t prmt_sel = static_cast<uint32_t>((g >> 2) | ((2 + (g >> 2)) << 4) | ((4 + (g >> 2)) << 8) |
                                                  ((6 + (g >> 2)) << 12));
  const int psh = 2 * (g & 3);
  bool alive = true;

  for (int p = p0; p < p1; ++p) {
    const int lp = p - p0;
    const int stage = lp % C::STAGES;
    const int buf = lp & 1;
    if (!mbar_wait(&full[stage], static_cast<uint32_t>((lp / C::STAGES) & 1), a.err)) alive = false;
    if (!__syncthreads_and(alive)) break;
    const uint8_t* cs = smem + stage * C::ST_BYTES;
    const uint8_t* rs = cs + C::ST_CODES;
    const float* ps = reinterpret_cast<const float*>(rs + C::ST_ROPE);
    const bool page_ok = bad[stage] == 0;
    const int tpos0 = p * kPage;

    // ---- QK^T for tokens 16*warp + g and + 8 -------------------------------------------
    const int ta = 16 * warp + g, tb = ta + 8;
    float acc[NG + 1][HN][4];
#pragma unroll
    for (int x = 0; x < NG + 1; ++x)
#pragma unroll
      for (int t = 0; t < HN; ++t)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[x][t][k] = 0.f;
#pragma unroll
    for (int ch = 0; ch < C::CODE_ROW / 16; ++ch) {
      const uint4 wa = *reinterpret_cast<const uint4*>(cs + swz<C::CODE_ROW>(ta, ch * 16));
      const uint4 wb = *reinterpret_cast<const uint4*>(cs + swz<C::CODE_ROW>(tb, ch * 16));
      const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const int m = ch * 4 + k4;
        const int gr = m / 8;
        const uint32_t sa = wav[k4] >> (4 * qi);
        const uint32_t sb = wbv[k4] >> (4 * qi);
        const uint32_t a0 = lop_and_or(sa, 0x00030003u, kMagic);
        const uint32_t a1 = lop_and_or(sb, 0x00030003u, kMagic);
        const uint32_t a2 = lop_and_or(sa, 0x000C000Cu, kMagic);
        const uint32_t a3 = lop_and_or(sb, 0x000C000Cu, kMagic);
#pragma unroll
        for (int t = 0; t < HN; ++t) {
          const uint16_t* qrow = qk + (8 * t + g) * C::QROW + 16 * m + 2 * qi;
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(qrow);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(qrow + 8);
          mma_bf16_16816(acc[gr][t], a0, a1, a2, a3, b0, b1);
        }
      }
    }
#pragma unroll
    for (int kk = 0; kk < C::KS_PE; ++kk) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(rs + swz<DR * 2>(ta, (16 * kk + 2 * qi) * 2));
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(rs + swz<DR * 2>(tb, (16 * kk + 2 * qi) * 2));
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(rs + swz<DR * 2>(ta, (16 * kk + 2 * qi + 8) * 2));
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(rs + swz<DR * 2>(tb, (16 * kk + 2 * qi + 8) * 2));
#pragma unroll
      for (int t = 0; t < HN; ++t) {
        const uint16_t* qrow = qk + (8 * t + g) * C::QROW + D + 16 * kk + 2 * qi;
        mma_bf16_16816(acc[NG][t], a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(qrow),
                       *reinterpret_cast<const uint32_t*>(qrow + 8));
      }
    }

    // ---- scores (log2 domain) and the tile max ------------------------------------------
    float sc[2][NG], ze[2][NG], zp[2][NG], s2[2][HN][2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int tok = rr ? tb : ta;
      const int pos = tpos0 + tok;
      const bool valid = page_ok && pos >= lo && pos < hi;
#pragma unroll
      for (int gr = 0; gr < NG; ++gr) {
        const float2 sz = reinterpret_cast<const float2*>(ps)[tok * NG + gr];
        sc[rr][gr] = sz.x;
        ze[rr][gr] = sz.y;
        zp[rr][gr] = sz.y;
      }
#pragma unroll
      for (int t = 0; t < HN; ++t)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          float s = acc[NG][t][rr * 2 + cc];
#pragma unroll
          for (int gr = 0; gr < NG; ++gr) {
            // scale * (acc - corr - zero * qsum), corr = the 128 / 32 offsets
            const float inner = fmaf(-ze[rr][gr], lqsum[gr][t][cc], acc[gr][t][rr * 2 + cc] - lcorr[gr][t][cc]);
            s = fmaf(sc[rr][gr], inner, s);
          }
          s2[rr][t][cc] = valid ? s * sl2 : -INFINITY;
        }
    }
#pragma unroll
    for (int t = 0; t < HN; ++t)
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float mx = fmaxf(s2[0][t][cc], s2[1][t][cc]);
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
        if (g == 0) red[(buf * 4 + warp) * H + 8 * t + 2 * qi + cc] = mx;
      }
    __syncthreads();
    if (tid == 0 && p + 2 < p1) issue(p + 2, (lp + 2) % C::STAGES);

    // ---- online softmax, P' = P * scale_g to smem, the zero-point correction ----------
    float alpha[HN][2];
#pragma unroll
    for (int t = 0; t < HN; ++t)
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int h = 8 * t + 2 * qi + cc;
        float mt = red[(buf * 4 + 0) * H + h];
#pragma unroll
        for (int w = 1; w < 4; ++w) mt = fmaxf(mt, red[(buf * 4 + w) * H + h]);
        const float mn = fmaxf(m_run[t][cc], mt);
        const float mref = mn == -INFINITY ? 0.f : mn;
        alpha[t][cc] = exp2f(m_run[t][cc] - mref);
        m_run[t][cc] = mn;
        const float pa = exp2f(s2[0][t][cc] - mref);
        const float pb = exp2f(s2[1][t][cc] - mref);
        s2[0][t][cc] = pa;
        s2[1][t][cc] = pb;
        l_part[t][cc] = fmaf(l_part[t][cc], alpha[t][cc], pa + pb);
      }
    uint16_t* pw = pbuf + buf * (NG * kPage * C::PSTRIDE);
#pragma unroll
    for (int gr = 0; gr < NG; ++gr)
#pragma unroll
      for (int t = 0; t < HN; ++t) {
        y_part[gr][t][0] *= alpha[t][0];
        y_part[gr][t][1] *= alpha[t][1];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int tok = rr ? tb : ta;
          // P' in FP16 (11-bit significand); the zero-point correction uses the same
          // rounded values the tensor cores multiply
          const __half2 ph = __floats2half2_rn(s2[rr][t][0] * sc[rr][gr], s2[rr][t][1] * sc[rr][gr]);
          *reinterpret_cast<__half2*>(pw + (gr * kPage + tok) * C::PSTRIDE + 8 * t + 2 * qi) = ph;
          const float2 pf = __half22float2(ph);
          y_part[gr][t][0] = fmaf(pf.x, zp[rr][gr], y_part[gr][t][0]);
          y_part[gr][t][1] = fmaf(pf.y, zp[rr][gr], y_part[gr][t][1]);
        }
      }
    __syncthreads();

    // ---- PV: O^T[e0 .. e0 + D/4) x heads ---------------------------------------------
    bool any_rescale = false;
#pragma unroll
    for (int t = 0; t < HN; ++t) any_rescale |= (alpha[t][0] != 1.f) | (alpha[t][1] != 1.f);
    if (__any_sync(0xFFFFFFFFu, any_rescale)) {
#pragma unroll
      for (int mt = 0; mt < C::MT; ++mt)
#pragma unroll
        for (int t = 0; t < HN; ++t) {
          o[mt][t][0] *= alpha[t][0];
          o[mt][t][1] *= alpha[t][1];
          o[mt][t][2] *= alpha[t][0];
          o[mt][t][3] *= alpha[t][1];
        }
    }
    const uint16_t* pg = pw + grw * kPage * C::PSTRIDE;
#pragma unroll
    for (int ks = 0; ks < kPage / 16; ++ks) {
      uint32_t bf[HN][2];
#pragma unroll
      for (int t = 0; t + 1 < HN; t += 2) {
        const uint32_t addr =
            smem_u32(pg + (16 * ks + (lane & 15)) * C::PSTRIDE + 8 * t + 8 * (lane >> 4));
        ldsm_x4_trans(addr, bf[t][0], bf[t][1], bf[t + 1][0], bf[t + 1][1]);
      }
      if (HN & 1) {
        const uint32_t addr = smem_u32(pg + (16 * ks + (lane & 15)) * C::PSTRIDE + 8 * (HN - 1));
        ldsm_x2_trans(addr, bf[HN - 1][0], bf[HN - 1][1]);
      }
      const int t0 = 16 * ks + 2 * qi;
      const int tok4[4] = {t0, t0 + 1, t0 + 8, t0 + 9};
      uint32_t wv[4][C::MT];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
#pragma unroll
        for (int c4 = 0; c4 < C::MT / 4; ++c4) {
          const uint4 w4 = *reinterpret_cast<const uint4*>(cs + swz<C::CODE_ROW>(tok4[x], e0 / 4 + c4 * 16));
          wv[x][c4 * 4 + 0] = w4.x;
          wv[x][c4 * 4 + 1] = w4.y;
          wv[x][c4 * 4 + 2] = w4.z;
          wv[x][c4 * 4 + 3] = w4.w;
        }
      }
#pragma unroll
      for (int mt = 0; mt < C::MT; ++mt) {
        const uint32_t r1 = prmt(wv[0][mt], wv[1][mt], prmt_sel);
        const uint32_t r2 = prmt(wv[2][mt], wv[3][mt], prmt_sel);
        // exact FP16 codes: (1024 + c) - 1024.  The offset must not reach the
        // accumulator, whose additions truncate: 1024 * sum(P') would swamp sum(P' c).
        const uint32_t a0 = hsub_magic16(lop_and_or(r1 >> psh, 0x00030003u, kMagic16));
        const uint32_t a1 = hsub_magic16(lop_and_or(r1 >> (psh + 8), 0x00030003u, kMagic16));
        const uint32_t a2 = hsub_magic16(lop_and_or(r2 >> psh, 0x00030003u, kMagic16));
        const uint32_t a3 = hsub_magic16(lop_and_or(r2 >> (psh + 8), 0x00030003u, kMagic16));
#pragma unroll
        for (int t = 0; t < HN; ++t) mma_f16_16816(o[mt][t], a0, a1, a2, a3, bf[t][0], bf[t][1]);
      }
    }
  }

  // ---- combine the per-lane partials and write this split's (lse, o) ----------------------
  __syncthreads();
  float* lred = red;  // [4][H]
#pragma unroll
  for (int t = 0; t < HN; ++t)
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      float l = l_part[t][cc];
      l += __shfl_xor_sync(0xFFFFFFFFu, l, 4);
      l += __shfl_xor_sync(0xFFFFFFFFu, l, 8);
      l += __shfl_xor_sync(0xFFFFFFFFu, l, 16);
      if (g == 0) lred[warp * H + 8 * t + 2 * qi + cc] = l;
#pragma unroll
      for (int gr = 0; gr < NG; ++gr) {
        float y = y_part[gr][t][cc];
        y += __shfl_xor_sync(0xFFFFFFFFu, y, 4);
        y += __shfl_xor_sync(0xFFFFFFFFu, y, 8);
        y += __shfl_xor_sync(0xFFFFFFFFu, y, 16);
        if (g == 0) yred[(warp * NG + gr) * H + 8 * t + 2 * qi + cc] = y;
      }
    }
  __syncthreads();
  float inv_l[HN][2], ytot[HN][2];
#pragma unroll
  for (int t = 0; t < HN; ++t)
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int h = 8 * t + 2 * qi + cc;
      float l = 0.f, y = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        l += lred[w * H + h];
        y += yred[(w * NG + grw) * H + h];
      }
      inv_l[t][cc] = l > 0.f ? 1.f / l : 0.f;
      ytot[t][cc] = y;
      if (warp == 0 && g == 0) {
        a.part_lse[(static_cast<int64_t>(b) * H + h) * S + split] =
            l > 0.f ? (m_run[t][cc] + __log2f(l)) * kLn2 : -INFINITY;
      }
    }
#pragma unroll
  for (int mt = 0; mt < C::MT; ++mt)
#pragma unroll
    for (int t = 0; t < HN; ++t)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int cc = k & 1;
        const int h = 8 * t + 2 * qi + cc;
        const int j = e0 + 16 * mt + g + (k >> 1) * 8;
        a.part_o[((static_cast<int64_t>(b) * H + h) * S + split) * D + j] =
            (o[mt][t][k] - ytot[t][cc]) * inv_l[t][cc];
      }
}

// ---- LSE merge of normalised partials -----------------------------------------------------

// One CTA per row.  The part weights exp(lse_p - m) / sum are computed once into shared
// memory; with VEC each thread then reads 4 consecutive elements of every part with 16-byte
// loads (all parts in flight at once) and writes 4 outputs (8-byte BF16 stores).
template <bool VEC>
__global__ void merge_kernel(const float* __restrict__ part_o, int64_t row_stride, int64_t part_stride,
                             const float* __restrict__ part_lse, int64_t lse_row_stride, int64_t lse_part_stride,
                             int n_parts, int d, uint16_t* __restrict__ out_bf16, float* __restrict__ out_f32,
                             int64_t ld_out, float* __restrict__ out_lse) {
  extern __shared__ float wts[];  // [n_parts]
  __shared__ float red[2];
  const int64_t row = blockIdx.x;
  const float* lse = part_lse + row * lse_row_stride;
  if (threadIdx.x < 32) {
    float m = -INFINITY;
    for (int p = threadIdx.x; p < n_parts; p += 32) m = fmaxf(m, lse[p * lse_part_stride]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    const float mref = m == -INFINITY ? 0.f : m;
    float den = 0.f;
    for (int p = threadIdx.x; p < n_parts; p += 32) {
      const float w = __expf(lse[p * lse_part_stride] - mref);
      wts[p] = w;
      den += w;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) den += __shfl_xor_sync(0xFFFFFFFFu, den, o);
    if (threadIdx.x == 0) {
      red[0] = mref;
      red[1] = den;
    }
  }
  __syncthreads();
  const float mref = red[0], den = red[1];
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const float* po = part_o + row * row_stride;
  if (VEC) {
    for (int j = 4 * threadIdx.x; j < d; j += 4 * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int p = 0; p < n_parts; ++p) {  // unconditional loads (all in flight); empty parts masked
        const float w = wts[p];
        const float4 v = *reinterpret_cast<const float4*>(po + p * part_stride + j);
        acc.x = w > 0.f ? fmaf(w, v.x, acc.x) : acc.x;
        acc.y = w > 0.f ? fmaf(w, v.y, acc.y) : acc.y;
        acc.z = w > 0.f ? fmaf(w, v.z, acc.z) : acc.z;
        acc.w = w > 0.f ? fmaf(w, v.w, acc.w) : acc.w;
      }
      acc.x *= inv;
      acc.y *= inv;
      acc.z *= inv;
      acc.w *= inv;
      if (out_f32) *reinterpret_cast<float4*>(out_f32 + row * ld_out + j) = acc;
      if (out_bf16) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        *reinterpret_cast<uint2*>(out_bf16 + row * ld_out + j) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
      }
    }
  } else {
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
      float acc = 0.f;
      for (int p = 0; p < n_parts; ++p) {
        const float w = wts[p];
        if (w > 0.f) acc = fmaf(w, po[p * part_stride + j], acc);
      }
      acc *= inv;
      if (out_f32) out_f32[row * ld_out + j] = acc;
      if (out_bf16) {
        const __nv_bfloat16 h = __float2bfloat16_rn(acc);
        out_bf16[row * ld_out + j] = *reinterpret_cast<const uint16_t*>(&h);
      }
    }
  }
  if (threadIdx.x == 0 && out_lse) out_lse[row] = den > 0.f ? mref + logf(den) : -INFINITY;
}

// Many partials (n_parts >= wide::kMinParts): a CTA per (row, 128-column chunk), its warps
// taking the partials in turn; rows, parts and outputs as merge_kernel<true> reads them.
__global__ void __launch_bounds__(wide::kThreads)
    merge_wide_kernel(const float* __restrict__ part_o, int64_t row_stride, int64_t part_stride,
                      const float* __restrict__ part_lse, int64_t lse_row_stride, int64_t lse_part_stride, int n_parts,
                      int d, uint16_t* __restrict__ out_bf16, float* __restrict__ out_f32, int64_t ld_out,
                      float* __restrict__ out_lse) {
  __shared__ float4 red[wide::kWarps][32];
  const int chunks = (d + wide::kCols - 1) / wide::kCols;
  const int64_t row = blockIdx.x / chunks;
  const int c0 = static_cast<int>(blockIdx.x % chunks) * wide::kCols;
  float4 res;
  const float lse = wide::merge_chunk(part_o + row * row_stride, part_stride, part_lse + row * lse_row_stride,
                                      lse_part_stride, n_parts, c0, d, red, res);
  if (threadIdx.x >= 32) return;
  const int col = c0 + 4 * threadIdx.x;
  if (col < d) {
    if (out_f32) *reinterpret_cast<float4*>(out_f32 + row * ld_out + col) = res;
    if (out_bf16) *reinterpret_cast<uint2*>(out_bf16 + row * ld_out + col) = wide::to_bf16x4(res);
  }
  if (c0 == 0 && threadIdx.x == 0 && out_lse) out_lse[row] = lse;
}

// Window split + LSE merge for the tcgen05 path, one CTA per (request, 4 heads), 256 threads.
//
// Phase 1 does not read the INT2 partials, so it runs while the tcgen05 kernel drains (this
// kernel is launched as its programmatic dependent): the window rows' slots and ring rows
// once per CTA; the rows staged in shared memory as FP32 with every load issued before any
// is used (the phase then costs a few round trips to memory, so that it finishes on the SMs
// the draining grid frees); scores with a warp pair per head (warp 2h + e takes rows e,
// e + 2, ..; lane l owns latent elements 4l + 128u + c and rope elements 4l + c); the window
// softmax (a warp per head); the window partial (thread: head tid / 64, elements
// 8 (tid % 64) ..+8), stored
// as split num_splits of part_o / part_lse so that the scratch holds every partial after the
// call.  Phase 2, after griddepcontrol.wait: each warp reads its head's split LSEs (lane =
// split; the weights reach the other lanes by shuffle) and merges the partials.
constexpr int kMwHeads = 4;
constexpr int kMwThreads = 256;
constexpr int kMwFastSplits = 12;  // up to this many INT2 splits, phase 2 issues all loads at once

template <int D, int DR>
__device__ __forceinline__ void window_elems4(const DecodeArgs& a, int64_t slot, int64_t r, int e0, float (&v)[4]) {
  if (r >= 0) {
    const uint2 w = *reinterpret_cast<const uint2*>(a.cache.hp + r * D + e0);
    v[0] = __uint_as_float(w.x << 16);
    v[1] = __uint_as_float(w.x & 0xFFFF0000u);
    v[2] = __uint_as_float(w.y << 16);
    v[3] = __uint_as_float(w.y & 0xFFFF0000u);
  } else {
    const uint32_t cb = a.cache.codes[slot * (D / 4) + e0 / 4];
    const float2 sz = reinterpret_cast<const float2*>(a.cache.params)[slot * (D / 128) + e0 / 128];
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = __fmul_rn(__fsub_rn(static_cast<float>((cb >> (2 * c)) & 3u), sz.y), sz.x);
  }
}

template <int D, int DR>
__global__ void __launch_bounds__(kMwThreads, 2) merge_window_kernel(const DecodeArgs a, int heads,
                                                                  uint16_t* __restrict__ out, int64_t out_sb,
                                                                  int64_t out_sh, float* __restrict__ out_lse) {
  static_assert(D == 4 * 128 && DR == 64, "four latent elements per lane, 16 rope lanes; 8 elements per thread");
  static_assert(kMwThreads == kMwHeads * (D / 8) && kMwThreads == 64 * kMwHeads, "thread <-> (head, elements)");
  __shared__ float sc[kMwHeads][kMaxWindow];
  __shared__ int64_t rslot[kMaxWindow], rrow[kMaxWindow];
  __shared__ float stat[kMwHeads][2];  // window lse, window sum of exp
  extern __shared__ float4 wrow_raw[];
  float* wrow = reinterpret_cast<float*>(wrow_raw);  // [nw][D + DR] FP32 window rows
  const int hgroups = heads / kMwHeads;
  const int b = blockIdx.x / hgroups, h0 = (blockIdx.x % hgroups) * kMwHeads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = a.num_splits + 1;
  int L = a.seq_lens[b];
  if (L < 0) L = 0;
  if (L > a.max_pages * kPage) L = a.max_pages * kPage;
  const int P = a.cache.sink, W = a.cache.recent;
  const int lo = min(P, L);
  const int hs = max(lo, L - W);
  int rs = 0, re = L;
  if (a.token_range != nullptr) {
    rs = max(0, a.token_range[2 * b]);
    re = min(L, a.token_range[2 * b + 1]);
  }
  const int s1 = min(max(rs, 0), lo), e1 = max(min(re, lo), s1);
  const int s2 = min(max(rs, hs), L), e2 = max(min(re, L), s2);
  const int n1 = e1 - s1;
  const int nw = n1 + (e2 - s2);  // <= sink + recent <= kMaxWindow (checked by the host)
  if (tid < nw) {
    const int pos = tid < n1 ? s1 + tid : s2 + (tid - n1);
    const int64_t page = a.page_table[b * a.pt_stride + pos / kPage];
    int64_t slot = -1, r = -1;
    if (page >= 0 && (page + 1) * kPage <= a.cache.num_slots) {
      slot = page * kPage + pos % kPage;
      r = a.cache.rows ? a.cache.rows[slot] : -1;
      if (!(r >= 0 && r < a.cache.num_ring_rows && a.cache.owners[r] == slot)) r = -1;
    } else {
      report(a.err, ROLAQ_DEV_BAD_PAGE);
    }
    rslot[tid] = slot;
    rrow[tid] = r;
  }
  __syncthreads();
  // The window rows into shared memory as FP32, (D + DR) values per row: every load of the
  // CTA is issued before any is used.  Latent elements come from the BF16 ring row, or (the
  // ring row no longer belongs to the slot) from the INT2 codes as (code - zero) * scale;
  // rope elements from k_pe; a row whose page is out of range stays zero.
  constexpr int kChunks = (D + DR) / 4;  // 4 values per chunk
  constexpr int kPerThread = (kMaxWindow * kChunks + kMwThreads - 1) / kMwThreads;
  {
    uint2 raw[kPerThread];
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
      const int idx = tid + k * kMwThreads;
      raw[k] = make_uint2(0, 0);
      if (idx < nw * kChunks) {
        const int p = idx / kChunks, e4 = 4 * (idx % kChunks);
        const int64_t slot = rslot[p], r = rrow[p];
        if (slot >= 0 && e4 >= D)
          raw[k] = *reinterpret_cast<const uint2*>(a.cache.rope + slot * DR + (e4 - D));
        else if (slot >= 0 && r >= 0)
          raw[k] = *reinterpret_cast<const uint2*>(a.cache.hp + r * D + e4);
      }
    }
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
      const int idx = tid + k * kMwThreads;
      if (idx < nw * kChunks) {
        const int p = idx / kChunks, e4 = 4 * (idx % kChunks);
        float v[4];
        if (rslot[p] >= 0 && e4 < D && rrow[p] < 0) {
          window_elems4<D, DR>(a, rslot[p], -1, e4, v);
        } else {
          v[0] = __uint_as_float(raw[k].x << 16);
          v[1] = __uint_as_float(raw[k].x & 0xFFFF0000u);
          v[2] = __uint_as_float(raw[k].y << 16);
          v[3] = __uint_as_float(raw[k].y & 0xFFFF0000u);
        }
        *reinterpret_cast<float4*>(wrow + p * (D + DR) + e4) = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
  }
  // the query of head h0 + hw at the lane's elements
  const int hw = warp >> 1, par = warp & 1;
  const uint16_t* qh = a.q + b * a.q_sb + (h0 + hw) * a.q_sh;
  float qv[16], qr[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint2 w = *reinterpret_cast<const uint2*>(qh + 4 * lane + 128 * u);
    qv[4 * u] = __uint_as_float(w.x << 16);
    qv[4 * u + 1] = __uint_as_float(w.x & 0xFFFF0000u);
    qv[4 * u + 2] = __uint_as_float(w.y << 16);
    qv[4 * u + 3] = __uint_as_float(w.y & 0xFFFF0000u);
  }
  {
    const uint2 w = lane < DR / 4 ? *reinterpret_cast<const uint2*>(qh + D + 4 * lane) : make_uint2(0, 0);
    qr[0] = __uint_as_float(w.x << 16);
    qr[1] = __uint_as_float(w.x & 0xFFFF0000u);
    qr[2] = __uint_as_float(w.y << 16);
    qr[3] = __uint_as_float(w.y & 0xFFFF0000u);
  }
  __syncthreads();
  // scores: a warp pair per head, rows p = par + 2 i, from shared memory
  for (int p = par; p < nw; p += 2) {
    float acc = 0.f;
    if (rslot[p] >= 0) {
      const float* wr = wrow + p * (D + DR);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 v = *reinterpret_cast<const float4*>(wr + 4 * lane + 128 * u);
        acc = fmaf(qv[4 * u], v.x, acc);
        acc = fmaf(qv[4 * u + 1], v.y, acc);
        acc = fmaf(qv[4 * u + 2], v.z, acc);
        acc = fmaf(qv[4 * u + 3], v.w, acc);
      }
      const float4 v = lane < DR / 4 ? *reinterpret_cast<const float4*>(wr + D + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
      acc = fmaf(qr[0], v.x, acc);
      acc = fmaf(qr[1], v.y, acc);
      acc = fmaf(qr[2], v.z, acc);
      acc = fmaf(qr[3], v.w, acc);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    // a row whose page is out of range takes no weight (the INT2 splits skip such tokens too)
    if (lane == 0) sc[hw][p] = rslot[p] >= 0 ? acc * a.sm_scale : -INFINITY;
  }
  __syncthreads();
  if (warp < kMwHeads) {  // window softmax of head h0 + warp
    const float x = lane < nw ? sc[warp][lane] : -INFINITY;
    float m = x;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    const float e = x != -INFINITY ? __expf(x - m) : 0.f;
    float l = e;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    if (lane < nw) sc[warp][lane] = e;
    if (lane == 0) {
      stat[warp][0] = l > 0.f ? m + logf(l) : -INFINITY;
      stat[warp][1] = l;
    }
  }
  __syncthreads();
  // window partial of head hh at elements j .. j + 7; rows past nw (up to a multiple of 4)
  // add 0 * 0
  const int hh = tid >> 6, j = 8 * (tid & 63);
  float ow[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) ow[c] = 0.f;
  const int nw4 = (nw + 3) & ~3;
  for (int p = 0; p < nw4; ++p) {
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float e = 0.f;
    if (p < nw) {
      e = sc[hh][p];
      if (rslot[p] >= 0) {
        const float4 v0 = *reinterpret_cast<const float4*>(wrow + p * (D + DR) + j);
        const float4 v1 = *reinterpret_cast<const float4*>(wrow + p * (D + DR) + j + 4);
        v[0] = v0.x, v[1] = v0.y, v[2] = v0.z, v[3] = v0.w, v[4] = v1.x, v[5] = v1.y, v[6] = v1.z, v[7] = v1.w;
      }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) ow[c] = fmaf(e, v[c], ow[c]);
  }
  const float lse_w = stat[hh][0];
  const float il = stat[hh][1] > 0.f ? 1.f / stat[hh][1] : 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) ow[c] *= il;
  const int64_t row = static_cast<int64_t>(b) * heads + h0 + hh;
  float* prow = a.part_o + row * S * D;
  {
    float4* dst = reinterpret_cast<float4*>(prow + static_cast<int64_t>(a.num_splits) * D + j);
    dst[0] = make_float4(ow[0], ow[1], ow[2], ow[3]);
    dst[1] = make_float4(ow[4], ow[5], ow[6], ow[7]);
  }
  if ((tid & 63) == 0) a.part_lse[row * S + a.num_splits] = lse_w;

  // ---- phase 2: the INT2 partials, written by the kernel this launch depends on ----
  grid_dependency_wait();
  const int ns = a.num_splits;
  const float* lse_row = a.part_lse + row * S;
  uint16_t* const orow = out + b * out_sb + (h0 + hh) * out_sh + j;  // 8-byte aligned rows
  if (ns <= kMwFastSplits) {
    // Every split's LSE and partial loaded before any is used (one round trip to L2); the
    // same operations in the same order as the general loop below.
    const float lv = lane < ns ? lse_row[lane] : -INFINITY;
    float4 v[kMwFastSplits][2];
#pragma unroll
    for (int p = 0; p < kMwFastSplits; ++p) {
      if (p < ns) {
        const float4* src = reinterpret_cast<const float4*>(prow + static_cast<int64_t>(p) * D + j);
        v[p][0] = src[0];
        v[p][1] = src[1];
      }
    }
    float m = fmaxf(lse_w, lv);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    const float mref = m == -INFINITY ? 0.f : m;
    const float ww = lse_w == -INFINITY ? 0.f : __expf(lse_w - mref);
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = ww * ow[c];
    const float wl = lane < ns ? __expf(lv - mref) : 0.f;  // weight of split lane
    float den = wl;
#pragma unroll
    for (int p = 0; p < kMwFastSplits; ++p) {
      if (p < ns) {  // uniform across the warp
        const float w = __shfl_sync(0xFFFFFFFFu, wl, p);
        const float vv[8] = {v[p][0].x, v[p][0].y, v[p][0].z, v[p][0].w, v[p][1].x, v[p][1].y, v[p][1].z, v[p][1].w};
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = w > 0.f ? fmaf(w, vv[c], acc[c]) : acc[c];
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) den += __shfl_xor_sync(0xFFFFFFFFu, den, o);
    den += ww;
    const float inv = den > 0.f ? 1.f / den : 0.f;
    uint32_t pk[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const __nv_bfloat162 v2 = __floats2bfloat162_rn(acc[2 * c] * inv, acc[2 * c + 1] * inv);
      pk[c] = *reinterpret_cast<const uint32_t*>(&v2);
    }
    reinterpret_cast<uint2*>(orow)[0] = make_uint2(pk[0], pk[1]);
    reinterpret_cast<uint2*>(orow)[1] = make_uint2(pk[2], pk[3]);
    if ((tid & 63) == 0 && out_lse) out_lse[row] = den > 0.f ? mref + logf(den) : -INFINITY;
    return;
  }
  float m = lse_w;
  for (int p = lane; p < ns; p += 32) m = fmaxf(m, lse_row[p]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  const float mref = m == -INFINITY ? 0.f : m;
  const float ww = lse_w == -INFINITY ? 0.f : __expf(lse_w - mref);
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = ww * ow[c];
  float den = 0.f;
  for (int pb = 0; pb < ns; pb += 32) {
    const int cnt = min(32, ns - pb);
    const float wl = lane < cnt ? __expf(lse_row[pb + lane] - mref) : 0.f;  // weight of split pb + lane
    den += wl;
    for (int q = 0; q < cnt; q += 4) {  // four splits' loads in flight at once
      float4 v[4][2];
      float w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        w[u] = __shfl_sync(0xFFFFFFFFu, wl, (q + u) & 31);
        if (q + u >= cnt) w[u] = 0.f;
        const float4* src =
            reinterpret_cast<const float4*>(prow + static_cast<int64_t>(pb + min(q + u, cnt - 1)) * D + j);
        v[u][0] = src[0];
        v[u][1] = src[1];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // empty splits (weight 0) are masked, not multiplied
        const float vv[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w, v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = w[u] > 0.f ? fmaf(w[u], vv[c], acc[c]) : acc[c];
      }
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) den += __shfl_xor_sync(0xFFFFFFFFu, den, o);
  den += ww;
  const float inv = den > 0.f ? 1.f / den : 0.f;
  uint32_t pk[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const __nv_bfloat162 v2 = __floats2bfloat162_rn(acc[2 * c] * inv, acc[2 * c + 1] * inv);
    pk[c] = *reinterpret_cast<const uint32_t*>(&v2);
  }
  reinterpret_cast<uint2*>(orow)[0] = make_uint2(pk[0], pk[1]);
  reinterpret_cast<uint2*>(orow)[1] = make_uint2(pk[2], pk[3]);
  if ((tid & 63) == 0 && out_lse) out_lse[row] = den > 0.f ? mref + logf(den) : -INFINITY;
}

// ---- host side ---------------------------------------------------------------------------

static int map_rows(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner_elems,
                    uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ROLAQ_ECUDA;
  cuuint64_t dims[2] = {inner_elems, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(inner_elems), box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ROLAQ_OK : ROLAQ_ECUDA;
}

template <int D, int DR, int H>
static int launch_decode_t(const DecodeArgs& a, cudaStream_t s) {
  using C = DecodeCfg<D, DR, H>;
  CUtensorMap mc, mr;
  int rc = map_rows(&mc, a.cache.codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, D / 4, a.cache.num_slots, D / 4, kPage);
  if (rc != ROLAQ_OK) return rc;
  rc = map_rows(&mr, a.cache.rope, CU_TENSOR_MAP_DATA_TYPE_UINT16, DR, a.cache.num_slots, DR * 2, kPage);
  if (rc != ROLAQ_OK) return rc;
  static const bool attr_ok =
      cudaFuncSetAttribute(decode_kernel<D, DR, H>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) ==
      cudaSuccess;
  if (!attr_ok) return ROLAQ_ECUDA;
  dim3 grid(a.num_splits + 1, a.batch);
  decode_kernel<D, DR, H><<<grid, kDecodeThreads, C::SMEM, s>>>(mc, mr, a);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

template <int D, int DR, int H>
static int launch_window_t(const DecodeArgs& a, cudaStream_t s) {
  static_assert(H % kWinHeads == 0, "heads per window CTA");
  constexpr size_t smem = window_rows_smem<D, DR>();
  static const bool attr_ok =
      cudaFuncSetAttribute(window_rows_kernel<D, DR, H>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
      cudaSuccess;
  if (!attr_ok) return ROLAQ_ECUDA;
  window_rows_kernel<D, DR, H><<<dim3(a.batch, H / kWinHeads), kWinHeads * 32, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

bool decode_tc_supported(const DecodeArgs& a, int heads);
int launch_decode_tc(const DecodeArgs& a, int heads, cudaStream_t s, bool dependent = false);
int launch_decode_windowed(const DecodeArgs& a, int heads, uint16_t* out, int64_t out_sb, int64_t out_sh,
                           float* out_lse, cudaStream_t s);
bool window_first_fits(const DecodeArgs& a);

int launch_decode(const DecodeArgs& a, int heads, cudaStream_t s) {
  const int d = a.cache.latent_dim, dr = a.cache.rope_dim;
  if (decode_tc_supported(a, heads)) {
    // tcgen05 kernel for the INT2 splits, the window split on its own
    int rc = launch_decode_tc(a, heads, s);
    if (rc != ROLAQ_OK) return rc;
    if (d == 512) return heads == 16 ? launch_window_t<512, 64, 16>(a, s) : launch_window_t<512, 64, 8>(a, s);
    return heads == 40 ? launch_window_t<256, 32, 40>(a, s) : launch_window_t<256, 32, 16>(a, s);
  }
  if (d == 512 && dr == 64 && heads == 16) return launch_decode_t<512, 64, 16>(a, s);
  if (d == 512 && dr == 64 && heads == 8) return launch_decode_t<512, 64, 8>(a, s);
  if (d == 256 && dr == 32 && heads == 40) return launch_decode_t<256, 32, 40>(a, s);
  if (d == 256 && dr == 32 && heads == 16) return launch_decode_t<256, 32, 16>(a, s);
  return ROLAQ_EUNSUPPORTED;
}

int launch_merge(const float* part_o, int64_t row_stride, int64_t part_stride, const float* part_lse,
                 int64_t lse_row_stride, int64_t lse_part_stride, int n_parts, int64_t rows, int d,
                 uint16_t* out_bf16, float* out_f32, int64_t ld_out, float* out_lse, cudaStream_t s) {
  if (rows == 0) return ROLAQ_OK;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = d % 4 == 0 && row_stride % 4 == 0 && part_stride % 4 == 0 && a16(part_o) &&
                   (out_f32 == nullptr || (a16(out_f32) && ld_out % 4 == 0)) &&
                   (out_bf16 == nullptr || ((reinterpret_cast<uintptr_t>(out_bf16) & 7u) == 0 && ld_out % 4 == 0));
  const int64_t wide_ctas = rows * ((d + wide::kCols - 1) / wide::kCols);
  if (vec && n_parts >= wide::kMinParts && wide_ctas <= 0x7FFFFFFF) {
    merge_wide_kernel<<<static_cast<unsigned>(wide_ctas), wide::kThreads, 0, s>>>(
        part_o, row_stride, part_stride, part_lse, lse_row_stride, lse_part_stride, n_parts, d, out_bf16, out_f32,
        ld_out, out_lse);
    return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
  }
  const int threads = d >= 512 ? 128 : 64;
  const size_t smem = size_t(n_parts) * sizeof(float);
  if (smem > 48 * 1024) return ROLAQ_EUNSUPPORTED;
  if (vec)
    merge_kernel<true><<<static_cast<unsigned>(rows), threads, smem, s>>>(
        part_o, row_stride, part_stride, part_lse, lse_row_stride, lse_part_stride, n_parts, d, out_bf16, out_f32,
        ld_out, out_lse);
  else
    merge_kernel<false><<<static_cast<unsigned>(rows), threads, smem, s>>>(
        part_o, row_stride, part_stride, part_lse, lse_row_stride, lse_part_stride, n_parts, d, out_bf16, out_f32,
        ld_out, out_lse);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

// tcgen05 INT2 splits + the fused window/merge kernel, when the shape and the output
// layout allow it (contiguous [B, H, D] partials, 8-byte aligned output rows); otherwise
// ROLAQ_EUNSUPPORTED and the caller runs launch_decode + launch_merge.
int launch_decode_merged(const DecodeArgs& a, int heads, uint16_t* out, int64_t out_sb, int64_t out_sh,
                         float* out_lse, cudaStream_t s) {
  if (!decode_tc_supported(a, heads)) return ROLAQ_EUNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) || (out_sb & 3) || (out_sh & 3) ||
      (reinterpret_cast<uintptr_t>(a.part_o) & 15u))
    return ROLAQ_EUNSUPPORTED;
  if (heads % kMwHeads != 0) return ROLAQ_EUNSUPPORTED;
  // When the INT2 grid and the window CTAs fit on the SMs together: the window split first,
  // on the SMs the grid leaves free, and the INT2 kernel and the merge as programmatic
  // dependents (B64 x 16K, 2 splits: 157.6 us per layer in the benchmark step, against 167.8
  // for the window split and merge after the INT2 kernel).  With several waves
  // the window CTAs would hold SMs the INT2 grid needs: for D = 512 the window split and the
  // merge then run in one dependent kernel after the INT2 kernel (below); for D = 256 the
  // caller takes the separate launches.
  if (window_first_fits(a)) return launch_decode_windowed(a, heads, out, out_sb, out_sh, out_lse, s);
  if (a.cache.latent_dim != 512) return ROLAQ_EUNSUPPORTED;
  // the merge kernel stages the window rows (at most sink + recent <= kMaxWindow) as FP32
  constexpr int kMwRowBytes = (512 + 64) * 4;
  static const bool mw_attr = cudaFuncSetAttribute(merge_window_kernel<512, 64>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   kMaxWindow * kMwRowBytes) == cudaSuccess;
  if (!mw_attr) return ROLAQ_ECUDA;
  int rc = launch_decode_tc(a, heads, s);
  if (rc != ROLAQ_OK) return rc;
  // Programmatic dependent launch: the window phase overlaps the tcgen05 kernel's last CTAs;
  // the merge waits for that grid's completion (griddepcontrol.wait) before reading partials.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(int64_t(a.batch) * heads / kMwHeads));
  cfg.blockDim = dim3(kMwThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(max(0, a.cache.sink + a.cache.recent)) * kMwRowBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, merge_window_kernel<512, 64>, a, heads, out, out_sb, out_sh, out_lse) != cudaSuccess)
    return ROLAQ_ECUDA;
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

}  // namespace rolaq
