// The window split and the final merge of the packed decode, as the two kernels around the
// tcgen05 INT2 kernel:
//
//   window_split_kernel  ->  decode_tc_kernel (programmatic dependent)  ->  merge_splits_kernel
//                                                                          (programmatic dependent)
//
// Reference behaviour: upstream _fwd_hp_window_stage1 and stage 2 of packed_mla_decode_gf_fwd
// (called at deployment/patches/rolaq_sglang.patch:98-111): the sink/recent tokens are
// attended from their BF16 ring rows (hp_c, owned by the slot) or, when the ring row has been
// taken over, from the INT2 codes; that window split and the INT2 splits are merged by
// log-sum-exp.
//
// The window split is a few dependent memory round trips per request (page -> slot -> ring
// row -> row), so it is given only the SMs the INT2 grid leaves free (used when that grid fits
// one wave): a CTA serves several requests (all heads), staging their window rows in shared
// memory as FP32, a chunk of requests at a time.  It lets the INT2 kernel launch at once
// (griddepcontrol.launch_dependents), so the INT2 CTAs fill every other SM while it runs.
// The merge kernel is launched as a dependent of the INT2 kernel: its CTAs are placed as the
// INT2 grid's last CTAs retire and wait (griddepcontrol.wait) for that grid, which itself
// waits for the window kernel before it exits.
#include "kernels.cuh"
#include "merge.cuh"

namespace rolaq {
namespace win {

constexpr int kMaxWindow = 32;  // sink + recent (checked by the host)
constexpr int THREADS = 512;
constexpr int kPage = 64;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
// four BF16 (packed in two words) -> FP32
__device__ __forceinline__ float4 bf16x4(uint2 w) {
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u), __uint_as_float(w.y << 16),
                     __uint_as_float(w.y & 0xFFFF0000u));
}
__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
  return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, fmaf(a.x, b.x, acc))));
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Window positions of request b: [s1, e1) u [s2, e2) (sink part, recent part), restricted
// to the request's token range; returns the row count.
__device__ __forceinline__ int window_rows(const DecodeArgs& a, int b, int& s1, int& n1, int& s2) {
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
  s1 = min(max(rs, 0), lo);
  const int e1 = max(min(re, lo), s1);
  s2 = min(max(rs, hs), L);
  const int e2 = max(min(re, L), s2);
  n1 = e1 - s1;
  return n1 + (e2 - s2);
}

// A CTA serves `per_cta` requests, `rpc` at a time.  Dynamic shared memory: FP32 rows
// [rpc][nwmax][D + DR], then slot and ring-row indices [rpc][kMaxWindow] (int64) and the row
// counts [rpc].
constexpr int kStageLoads = 12;  // staged 16-byte row pieces per thread and chunk (host-checked)

template <int D, int DR, int H>
__global__ void __launch_bounds__(THREADS, 1) window_split_kernel(const DecodeArgs a, int rpc, int per_cta) {
  constexpr int KW = D + DR;
  extern __shared__ float4 smem4[];
  const int nwmax = a.cache.sink + a.cache.recent;
  float* rows = reinterpret_cast<float*>(smem4);
  int64_t* rslot = reinterpret_cast<int64_t*>(rows + size_t(rpc) * nwmax * KW);
  int64_t* rrow = rslot + rpc * kMaxWindow;
  int* nwv = reinterpret_cast<int*>(rrow + rpc * kMaxWindow);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) grid_launch_dependents();  // the INT2 kernel may start on the other SMs now
  const int S = a.num_splits + 1;
  const int bend = min(a.batch, (blockIdx.x + 1) * per_cta);
  // the CTA's requests, rpc at a time
  for (int b0 = blockIdx.x * per_cta; b0 < bend; b0 += rpc) {
  if (b0 > blockIdx.x * per_cta) __syncthreads();  // the previous chunk's rows are no longer read

  // -- per (request, row): slot and the ring row that holds it (if it still belongs to it) --
  for (int idx = tid; idx < rpc * kMaxWindow; idx += THREADS) {
    const int r = idx / kMaxWindow, p = idx % kMaxWindow, b = b0 + r;
    int64_t slot = -1, rr = -1;
    if (b < bend) {
      int s1, n1, s2;
      const int nw = window_rows(a, b, s1, n1, s2);
      if (p == 0) nwv[r] = nw;
      if (p < nw) {
        const int pos = p < n1 ? s1 + p : s2 + (p - n1);
        const int64_t page = a.page_table[b * a.pt_stride + pos / kPage];
        if (page >= 0 && (page + 1) * kPage <= a.cache.num_slots) {
          slot = page * kPage + pos % kPage;
          rr = a.cache.rows ? a.cache.rows[slot] : -1;
          if (!(rr >= 0 && rr < a.cache.num_ring_rows && a.cache.owners[rr] == slot)) rr = -1;
        } else {
          report(a.err, ROLAQ_DEV_BAD_PAGE);
        }
      }
    } else if (p == 0) {
      nwv[r] = 0;
    }
    rslot[idx] = slot;
    rrow[idx] = rr;
  }
  __syncthreads();
  // -- the rows into shared memory as FP32, eight values per thread and step: latent values
  //    from the BF16 ring row or (ring row taken over) (code - zero) * scale, rope values
  //    from k_pe; absent rows stay zero --
  constexpr int C8 = KW / 8;
  static_assert(KW % 8 == 0 && D % 8 == 0, "16-byte row pieces");
  {
    // every load of the thread is issued before any is used (one round trip per chunk)
    const int total = rpc * nwmax * C8;
    uint4 raw[kStageLoads];
#pragma unroll
    for (int k = 0; k < kStageLoads; ++k) {
      const int idx = tid + k * THREADS;
      raw[k] = make_uint4(0, 0, 0, 0);
      if (idx < total) {
        const int row = idx / C8, e8 = 8 * (idx % C8), r = row / nwmax, p = row % nwmax;
        const int64_t slot = rslot[r * kMaxWindow + p], rr = rrow[r * kMaxWindow + p];
        if (p < nwv[r] && slot >= 0) {
          if (e8 >= D)
            raw[k] = *reinterpret_cast<const uint4*>(a.cache.rope + slot * DR + (e8 - D));
          else if (rr >= 0)
            raw[k] = *reinterpret_cast<const uint4*>(a.cache.hp + rr * D + e8);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kStageLoads; ++k) {
      const int idx = tid + k * THREADS;
      if (idx >= total) continue;
      const int row = idx / C8, e8 = 8 * (idx % C8), r = row / nwmax, p = row % nwmax;
      const int64_t slot = rslot[r * kMaxWindow + p], rr = rrow[r * kMaxWindow + p];
      float4 v[2];
      if (p < nwv[r] && slot >= 0 && e8 < D && rr < 0) {  // ring row taken over (rare): the INT2 codes
        const uint32_t cw = *reinterpret_cast<const uint16_t*>(a.cache.codes + slot * (D / 4) + e8 / 4);
        const float2 sz = reinterpret_cast<const float2*>(a.cache.params)[slot * (D / 128) + e8 / 128];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const uint32_t cb = cw >> (8 * h2);
          v[h2] = make_float4(__fmul_rn(__fsub_rn(static_cast<float>(cb & 3u), sz.y), sz.x),
                              __fmul_rn(__fsub_rn(static_cast<float>((cb >> 2) & 3u), sz.y), sz.x),
                              __fmul_rn(__fsub_rn(static_cast<float>((cb >> 4) & 3u), sz.y), sz.x),
                              __fmul_rn(__fsub_rn(static_cast<float>((cb >> 6) & 3u), sz.y), sz.x));
        }
      } else {  // BF16 (ring row or k_pe); absent rows stay zero
        const uint4 w = raw[k];
        v[0] = make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u), __uint_as_float(w.y << 16),
                           __uint_as_float(w.y & 0xFFFF0000u));
        v[1] = make_float4(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xFFFF0000u), __uint_as_float(w.w << 16),
                           __uint_as_float(w.w & 0xFFFF0000u));
      }
      float4* dst = reinterpret_cast<float4*>(rows) + (size_t(r) * nwmax + p) * (KW / 4) + e8 / 4;
      dst[0] = v[0];
      dst[1] = v[1];
    }
  }
  __syncthreads();
  // -- a warp per (request, HB heads): lane l holds the latent float4 chunks l + 32 j and the
  //    rope chunk l (l < DR / 4) of every row, so that a warp's row read is 512 contiguous
  //    bytes (no bank conflicts) and serves HB heads; scores by warp sums, softmax over the
  //    rows (lane p holds row p), the window partials --
  constexpr int HB = D == 512 ? 2 : 4;  // heads per warp
  constexpr int NCH = D / 128;          // latent float4 chunks per lane
  constexpr int RCH = DR / 4;           // rope float4 chunks (lanes 0 .. RCH - 1)
  static_assert(H % HB == 0 && RCH <= 32, "head blocks, rope lanes");
  for (int item = warp; item < rpc * (H / HB); item += THREADS / 32) {
    const int r = item / (H / HB), h0 = (item % (H / HB)) * HB, b = b0 + r;
    if (b >= bend) continue;
    const int nw = nwv[r];
    float4 qv[HB][NCH], qr[HB];
#pragma unroll
    for (int hb = 0; hb < HB; ++hb) {
      const uint16_t* qh = a.q + b * a.q_sb + (h0 + hb) * a.q_sh;
#pragma unroll
      for (int j = 0; j < NCH; ++j) qv[hb][j] = bf16x4(*reinterpret_cast<const uint2*>(qh + 4 * (lane + 32 * j)));
      qr[hb] = lane < RCH ? bf16x4(*reinterpret_cast<const uint2*>(qh + D + 4 * lane)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float4* rbase = reinterpret_cast<const float4*>(rows + size_t(r) * nwmax * KW);
    float sp[HB];  // lane p: the score of row p
#pragma unroll
    for (int hb = 0; hb < HB; ++hb) sp[hb] = -INFINITY;
    // four rows at a time: their warp sums are independent shuffle chains (rows past nw are
    // zero in shared memory and their scores are dropped; the row index is clamped so that no
    // read leaves this request's rows)
    for (int p0 = 0; p0 < nw; p0 += 4) {
      float acc[4][HB];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4* rw = rbase + size_t(min(p0 + u, nwmax - 1)) * (KW / 4);
        float4 v[NCH];
#pragma unroll
        for (int j = 0; j < NCH; ++j) v[j] = rw[lane + 32 * j];
        const float4 vr = lane < RCH ? rw[D / 4 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int hb = 0; hb < HB; ++hb) {
          float t = dot4(qr[hb], vr, 0.f);
#pragma unroll
          for (int j = 0; j < NCH; ++j) t = dot4(qv[hb][j], v[j], t);
          acc[u][hb] = t;
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int hb = 0; hb < HB; ++hb) acc[u][hb] += __shfl_xor_sync(0xFFFFFFFFu, acc[u][hb], o);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int p = p0 + u;
        if (p >= nw) break;
        // a row whose page is out of range takes no weight (the INT2 splits skip such tokens too)
        const bool valid = rslot[r * kMaxWindow + p] >= 0;
#pragma unroll
        for (int hb = 0; hb < HB; ++hb)
          if (lane == p) sp[hb] = valid ? acc[u][hb] * a.sm_scale : -INFINITY;
      }
    }
    float e[HB], l[HB], m[HB];
#pragma unroll
    for (int hb = 0; hb < HB; ++hb) {
      m[hb] = warp_max(sp[hb]);
      e[hb] = sp[hb] != -INFINITY ? __expf(sp[hb] - m[hb]) : 0.f;
      l[hb] = warp_sum(e[hb]);
    }
    float4 o[HB][NCH];
#pragma unroll
    for (int hb = 0; hb < HB; ++hb)
#pragma unroll
      for (int j = 0; j < NCH; ++j) o[hb][j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int p = 0; p < nw; ++p) {
      const float4* rw = rbase + size_t(p) * (KW / 4);
      float4 v[NCH];
#pragma unroll
      for (int j = 0; j < NCH; ++j) v[j] = rw[lane + 32 * j];
#pragma unroll
      for (int hb = 0; hb < HB; ++hb) {
        const float w = __shfl_sync(0xFFFFFFFFu, e[hb], p);
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          o[hb][j].x = fmaf(w, v[j].x, o[hb][j].x);
          o[hb][j].y = fmaf(w, v[j].y, o[hb][j].y);
          o[hb][j].z = fmaf(w, v[j].z, o[hb][j].z);
          o[hb][j].w = fmaf(w, v[j].w, o[hb][j].w);
        }
      }
    }
#pragma unroll
    for (int hb = 0; hb < HB; ++hb) {
      const float il = l[hb] > 0.f ? 1.f / l[hb] : 0.f;
      const int64_t row = (static_cast<int64_t>(b) * H + h0 + hb) * S + a.num_splits;
      float4* dst = reinterpret_cast<float4*>(a.part_o + row * D);
#pragma unroll
      for (int j = 0; j < NCH; ++j)
        dst[lane + 32 * j] = make_float4(o[hb][j].x * il, o[hb][j].y * il, o[hb][j].z * il, o[hb][j].w * il);
      if (lane == 0) a.part_lse[row] = l[hb] > 0.f ? m[hb] + logf(l[hb]) : -INFINITY;
    }
  }
  }  // chunk
}

// The LSE merge of a request's num_splits + 1 partials (INT2 splits, window split last):
// one CTA per (request, 4 heads), D / 8 threads per head, 8 elements per thread.
template <int D>
__global__ void __launch_bounds__(4 * D / 8) merge_splits_kernel(const DecodeArgs a, int heads,
                                                                uint16_t* __restrict__ out, int64_t out_sb,
                                                                int64_t out_sh, float* __restrict__ out_lse) {
  constexpr int TPH = D / 8;  // threads per head (a multiple of 32)
  const int hgroups = heads / 4;
  const int b = blockIdx.x / hgroups, h = (blockIdx.x % hgroups) * 4 + threadIdx.x / TPH;
  const int j = 8 * (threadIdx.x % TPH), lane = threadIdx.x & 31;
  const int S = a.num_splits + 1;
  grid_dependency_wait();  // the INT2 kernel (and through it the window kernel) has completed
  const int64_t row = static_cast<int64_t>(b) * heads + h;
  const float* lse_row = a.part_lse + row * S;
  const float* prow = a.part_o + row * S * D + j;
  float m = -INFINITY;
  for (int p = lane; p < S; p += 32) m = fmaxf(m, lse_row[p]);
  m = warp_max(m);
  const float mref = m == -INFINITY ? 0.f : m;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.f;
  float den = 0.f;
  for (int pb = 0; pb < S; pb += 32) {
    const int cnt = min(32, S - pb);
    const float lv = lane < cnt ? lse_row[pb + lane] : -INFINITY;
    const float wl = lv != -INFINITY ? __expf(lv - mref) : 0.f;  // weight of split pb + lane
    den += wl;
    for (int q = 0; q < cnt; q += 4) {  // four splits' loads in flight at once
      float4 v[4][2];
      float w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        w[u] = __shfl_sync(0xFFFFFFFFu, wl, (q + u) & 31);
        if (q + u >= cnt) w[u] = 0.f;
        const float4* src = reinterpret_cast<const float4*>(prow + static_cast<int64_t>(pb + min(q + u, cnt - 1)) * D);
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
  den = warp_sum(den);
  const float inv = den > 0.f ? 1.f / den : 0.f;
  uint32_t pk[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const __nv_bfloat162 v2 = __floats2bfloat162_rn(acc[2 * c] * inv, acc[2 * c + 1] * inv);
    pk[c] = *reinterpret_cast<const uint32_t*>(&v2);
  }
  uint16_t* orow = out + b * out_sb + h * out_sh + j;
  reinterpret_cast<uint2*>(orow)[0] = make_uint2(pk[0], pk[1]);
  reinterpret_cast<uint2*>(orow)[1] = make_uint2(pk[2], pk[3]);
  if (threadIdx.x % TPH == 0 && out_lse) out_lse[row] = den > 0.f ? mref + logf(den) : -INFINITY;
}

// The same merge for many splits (num_splits + 1 >= wide::kMinParts): a CTA per (request,
// head, 128-column chunk), its warps taking the splits in turn.
template <int D>
__global__ void __launch_bounds__(wide::kThreads) merge_splits_wide_kernel(const DecodeArgs a, int heads,
                                                                           uint16_t* __restrict__ out, int64_t out_sb,
                                                                           int64_t out_sh, float* __restrict__ out_lse) {
  __shared__ float4 red[wide::kWarps][32];
  constexpr int CH = D / wide::kCols;
  const int64_t row = blockIdx.x / CH;  // b * heads + h
  const int c0 = (blockIdx.x % CH) * wide::kCols;
  const int S = a.num_splits + 1;
  grid_dependency_wait();  // the INT2 kernel (and through it the window kernel) has completed
  float4 res;
  const float lse = wide::merge_chunk(a.part_o + row * S * D, D, a.part_lse + row * S, 1, S, c0, D, red, res);
  if (threadIdx.x >= 32) return;
  const int64_t b = row / heads, h = row % heads;
  reinterpret_cast<uint2*>(out + b * out_sb + h * out_sh + c0)[threadIdx.x] = wide::to_bf16x4(res);
  if (c0 == 0 && threadIdx.x == 0 && out_lse) out_lse[row] = lse;
}

}  // namespace win

// Window split (normal launch), then the INT2 kernel and the merge as programmatic
// dependents.  Shapes and output alignment are checked by the caller.
int launch_decode_tc(const DecodeArgs& a, int heads, cudaStream_t s, bool dependent);
bool decode_tc_supported(const DecodeArgs& a, int heads);

// Requests per window CTA (rpc): as many as shared memory and the per-thread staging
// registers allow.
static int window_rpc(int d, int dr, int nwmax) {
  if (nwmax <= 0) return 8;
  const size_t per_req = size_t(nwmax) * (d + dr) * 4 + 2 * win::kMaxWindow * 8 + 4;
  int rpc = static_cast<int>((200 * 1024) / per_req);
  rpc = min(rpc, (win::kStageLoads * win::THREADS) / (nwmax * (d + dr) / 8));
  return max(1, min(rpc, 8));
}

// The window-first launch applies when the INT2 grid is one wave and leaves SMs free for the
// window CTAs, each looping over at most two chunks of rpc requests: the window grid then
// stays shorter than the INT2 kernel (B128 x 8K, D = 512, 1 split: 20 window CTAs, two chunks
// each: 176 against 188 us per layer for the window split after the INT2 kernel).
bool window_first_fits(const DecodeArgs& a) {
  const int rpc = window_rpc(a.cache.latent_dim, a.cache.rope_dim, a.cache.sink + a.cache.recent);
  const int64_t free_sms = sm_count() - int64_t(a.batch) * a.num_splits;
  return free_sms >= 1 && free_sms * 2 * rpc >= a.batch;
}

// CTAs: at most max_ctas (the SMs the INT2 grid leaves free: its CTAs hold a whole SM each),
// each looping over its requests rpc at a time.
template <int D, int DR, int H>
static int launch_window_split(const DecodeArgs& a, int max_ctas, cudaStream_t s) {
  const int nwmax = a.cache.sink + a.cache.recent;
  const size_t per_req = size_t(nwmax) * (D + DR) * 4 + 2 * win::kMaxWindow * 8 + 4;
  const int rpc = window_rpc(D, DR, nwmax);
  const int ctas = max(1, min((a.batch + rpc - 1) / rpc, max_ctas));
  const int per_cta = (a.batch + ctas - 1) / ctas;
  const int rpc_run = min(rpc, per_cta);  // a chunk never covers more requests than the CTA serves
  const size_t smem = size_t(rpc_run) * per_req + 16;
  static const bool attr = cudaFuncSetAttribute(win::window_split_kernel<D, DR, H>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)(208 * 1024)) == cudaSuccess;
  if (!attr) return ROLAQ_ECUDA;
  win::window_split_kernel<D, DR, H><<<static_cast<unsigned>(ctas), win::THREADS, smem, s>>>(a, rpc_run, per_cta);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

template <int D>
static int launch_merge_splits(const DecodeArgs& a, int heads, uint16_t* out, int64_t out_sb, int64_t out_sh,
                               float* out_lse, cudaStream_t s) {
  const bool many = a.num_splits + 1 >= wide::kMinParts;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(many ? int64_t(a.batch) * heads * (D / wide::kCols)
                                                : int64_t(a.batch) * heads / 4));
  cfg.blockDim = dim3(many ? wide::kThreads : 4 * D / 8);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      many ? cudaLaunchKernelEx(&cfg, win::merge_splits_wide_kernel<D>, a, heads, out, out_sb, out_sh, out_lse)
           : cudaLaunchKernelEx(&cfg, win::merge_splits_kernel<D>, a, heads, out, out_sb, out_sh, out_lse);
  if (e != cudaSuccess) return ROLAQ_ECUDA;
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

// The window split on win_ctas CTAs, then the INT2 kernel (grid as `a` says) and the merge as
// programmatic dependents.
static int launch_window_first(const DecodeArgs& a, int win_ctas, int heads, uint16_t* out, int64_t out_sb,
                               int64_t out_sh, float* out_lse, cudaStream_t s) {
  const int d = a.cache.latent_dim;
  int rc;
  if (d == 512)
    rc = heads == 16 ? launch_window_split<512, 64, 16>(a, win_ctas, s)
                     : launch_window_split<512, 64, 8>(a, win_ctas, s);
  else
    rc = heads == 40 ? launch_window_split<256, 32, 40>(a, win_ctas, s)
                     : launch_window_split<256, 32, 16>(a, win_ctas, s);
  if (rc != ROLAQ_OK) return rc;
  rc = launch_decode_tc(a, heads, s, true);
  if (rc != ROLAQ_OK) return rc;
  return d == 512 ? launch_merge_splits<512>(a, heads, out, out_sb, out_sh, out_lse, s)
                  : launch_merge_splits<256>(a, heads, out, out_sb, out_sh, out_lse, s);
}

// The split partials only (no merge): the window split first on the SMs a one-wave INT2 grid
// leaves free, the INT2 kernel as its programmatic dependent; else the INT2 kernel and the
// window split one after the other.
int launch_decode(const DecodeArgs& a, int heads, cudaStream_t s);
int launch_decode_partials(const DecodeArgs& a, int heads, cudaStream_t s) {
  if (!decode_tc_supported(a, heads) || !window_first_fits(a)) return launch_decode(a, heads, s);
  const int d = a.cache.latent_dim;
  const int win_ctas = max(1, sm_count() - a.batch * a.num_splits);
  int rc;
  if (d == 512)
    rc = heads == 16 ? launch_window_split<512, 64, 16>(a, win_ctas, s)
                     : launch_window_split<512, 64, 8>(a, win_ctas, s);
  else
    rc = heads == 40 ? launch_window_split<256, 32, 40>(a, win_ctas, s)
                     : launch_window_split<256, 32, 16>(a, win_ctas, s);
  if (rc != ROLAQ_OK) return rc;
  return launch_decode_tc(a, heads, s, true);
}

int launch_decode_windowed(const DecodeArgs& a, int heads, uint16_t* out, int64_t out_sb, int64_t out_sh,
                           float* out_lse, cudaStream_t s) {
  return launch_window_first(a, max(1, sm_count() - a.batch * a.num_splits), heads, out, out_sb, out_sh, out_lse, s);
}


}  // namespace rolaq
