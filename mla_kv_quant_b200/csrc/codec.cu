// SIMT kernels around the codec: scatter-pack of already-rotated FP32 rows, the
// writer's auxiliary stores, row dequantisation and the split-count preparation.
//
// References: scatter_pack_rows (deployment/patches/rolaq_sglang.patch:9-34),
// _aux (deployment/sglang/QuantKernel/mla_fused_writer.py:16-51),
// prepare_gf_splits (deployment/patches/rolaq_sglang.patch:81-92),
// affine dequant (mla_quant/oscar.py:144).
#include "kernels.cuh"

namespace rolaq {

// One thread per (row, 128-element group).  The three passes re-read the group's
// 512 bytes from L1/L2; the order of the FP32 sums is GroupSum's.
__global__ void scatter_pack_kernel(const float* __restrict__ x, int64_t ldx, const void* slots, int slots64,
                                    int64_t n, int d, rolaq_codec codec, uint8_t* __restrict__ codes,
                                    float* __restrict__ params, int64_t num_slots, int32_t* err) {
  const int ng = d / 128;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (unit >= n * ng) return;
  const int64_t row = unit / ng;
  const int g = static_cast<int>(unit % ng);
  const int64_t slot = load_index(slots, slots64, row);
  if (slot < 0 || slot >= num_slots) {
    report(err, ROLAQ_DEV_BAD_SLOT);
    return;
  }
  const float4* v = reinterpret_cast<const float4*>(x + row * ldx + g * 128);
  if (codec.family == ROLAQ_CODEC_UNIFORM) {  // OSCAR's uniform min/max codec
    float mn = INFINITY, mx = -INFINITY;
    for (int c = 0; c < 32; ++c) {
      const float4 q = v[c];
      mn = fminf(fminf(mn, q.x), fminf(fminf(q.y, q.z), q.w));
      mx = fmaxf(fmaxf(mx, q.x), fmaxf(fmaxf(q.y, q.z), q.w));
    }
    const float scale = uniform_scale(mn, mx);
    uint4* cdst = reinterpret_cast<uint4*>(codes + slot * (d / 4) + g * 32);
    uint32_t words[8];
    for (int w = 0; w < 8; ++w) {
      uint32_t word = 0;
      for (int j = 0; j < 4; ++j) {
        const float4 q = v[w * 4 + j];
        const int b = 8 * j;
        word |= uniform_code(q.x, mn, scale) << (b + 0);
        word |= uniform_code(q.y, mn, scale) << (b + 2);
        word |= uniform_code(q.z, mn, scale) << (b + 4);
        word |= uniform_code(q.w, mn, scale) << (b + 6);
      }
      words[w] = word;
    }
    cdst[0] = make_uint4(words[0], words[1], words[2], words[3]);
    cdst[1] = make_uint4(words[4], words[5], words[6], words[7]);
    reinterpret_cast<float2*>(params)[slot * ng + g] = make_float2(scale, uniform_zero(mn, scale));
    return;
  }
  GroupSum acc;
  acc.zero();
  for (int c = 0; c < 32; ++c) {
    const float4 q = v[c];
    const int k = (c & 1) * 4;
    acc.add(k + 0, q.x);
    acc.add(k + 1, q.y);
    acc.add(k + 2, q.z);
    acc.add(k + 3, q.w);
  }
  const float mean = __fmul_rn(acc.total(), 1.0f / 128.0f);
  acc.zero();
  for (int c = 0; c < 32; ++c) {
    const float4 q = v[c];
    const int k = (c & 1) * 4;
    float df;
    df = __fsub_rn(q.x, mean);
    acc.add(k + 0, __fmul_rn(df, df));
    df = __fsub_rn(q.y, mean);
    acc.add(k + 1, __fmul_rn(df, df));
    df = __fsub_rn(q.z, mean);
    acc.add(k + 2, __fmul_rn(df, df));
    df = __fsub_rn(q.w, mean);
    acc.add(k + 3, __fmul_rn(df, df));
  }
  const float var = __fmul_rn(acc.total(), 1.0f / 128.0f);
  const float stdv = __fsqrt_rn(__fadd_rn(var, 1e-8f));
  uint32_t words[8];
  for (int w = 0; w < 8; ++w) {
    uint32_t word = 0;
    for (int j = 0; j < 4; ++j) {
      const float4 q = v[w * 4 + j];
      const int b = 8 * j;
      word |= lloyd_code(__fsub_rn(q.x, mean), stdv, codec.threshold) << (b + 0);
      word |= lloyd_code(__fsub_rn(q.y, mean), stdv, codec.threshold) << (b + 2);
      word |= lloyd_code(__fsub_rn(q.z, mean), stdv, codec.threshold) << (b + 4);
      word |= lloyd_code(__fsub_rn(q.w, mean), stdv, codec.threshold) << (b + 6);
    }
    words[w] = word;
  }
  const float scale = __fmul_rn(codec.scale_factor, stdv);
  const float zero = __fsub_rn(codec.zero_const, __fdiv_rn(mean, scale));
  uint4* cdst = reinterpret_cast<uint4*>(codes + slot * (d / 4) + g * 32);
  cdst[0] = make_uint4(words[0], words[1], words[2], words[3]);
  cdst[1] = make_uint4(words[4], words[5], words[6], words[7]);
  reinterpret_cast<float2*>(params)[slot * ng + g] = make_float2(scale, zero);
}

// One warp per row: k_pe copy, ring row and slot <-> ring maps.
__global__ void aux_kernel(const float* __restrict__ c, int64_t ldc, const uint16_t* __restrict__ k_pe,
                           int64_t ld_pe, const int64_t* __restrict__ slots, const void* seq_lens, int seq64,
                           const void* req_idx, int req64, const void* positions, int pos64, int64_t n,
                           rolaq_layer_cache cache, int32_t* err) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const int64_t slot = slots[row];
  if (slot < 0 || slot >= cache.num_slots) {
    if (lane == 0) report(err, ROLAQ_DEV_BAD_SLOT);
    return;
  }
  if (slot == 0) return;  // slot 0 backs CUDA-graph padding
  for (int j = lane; j < cache.rope_dim; j += 32) cache.rope[slot * cache.rope_dim + j] = k_pe[row * ld_pe + j];
  if (seq_lens == nullptr || req_idx == nullptr || cache.rows == nullptr) return;
  const int P = cache.sink, W = cache.recent;
  const int64_t seq = load_index(seq_lens, seq64, row);
  const int64_t req = load_index(req_idx, req64, row);
  const int64_t pos = positions ? load_index(positions, pos64, row) : seq - 1;
  const bool keep = (P + W) > 0 && (pos < P || pos >= seq - W) && req >= 0 && req < cache.max_reqs && pos >= 0;
  int64_t ring = -1;
  if (keep) {
    const int64_t w = W > 0 ? W : 1;
    const int64_t inner = pos < P ? pos : P + ((pos - P) > 0 ? (pos - P) : 0) % w;
    ring = 1 + req * (P + W) + inner;
    if (ring >= cache.num_ring_rows) ring = -1;
  }
  if (ring >= 0) {
    for (int j = lane; j < cache.latent_dim; j += 32) {
      const __nv_bfloat16 h = __float2bfloat16_rn(c[row * ldc + j]);
      cache.hp[ring * cache.latent_dim + j] = *reinterpret_cast<const uint16_t*>(&h);
    }
  }
  if (lane == 0) {
    cache.rows[slot] = static_cast<int32_t>(ring);
    if (ring >= 0) cache.owners[ring] = static_cast<int32_t>(slot);
  }
}

// One thread per packed byte (4 latent elements).
__global__ void dequant_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ params,
                               const void* slots, int slots64, int64_t n, int d, int64_t num_slots,
                               float* __restrict__ out_f32, uint16_t* __restrict__ out_bf16, int64_t ld_out,
                               int32_t* err) {
  const int bpr = d / 4;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (unit >= n * bpr) return;
  const int64_t row = unit / bpr;
  const int b = static_cast<int>(unit % bpr);
  const int64_t slot = slots ? load_index(slots, slots64, row) : row;
  if (slot < 0 || slot >= num_slots) {
    if (b == 0) report(err, ROLAQ_DEV_BAD_SLOT);
    return;
  }
  const uint32_t byte = codes[slot * bpr + b];
  const int g = (4 * b) / 128;
  const float2 sz = reinterpret_cast<const float2*>(params)[slot * (d / 128) + g];
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = __fmul_rn(__fsub_rn(static_cast<float>((byte >> (2 * k)) & 3u), sz.y), sz.x);
  }
  if (out_f32) *reinterpret_cast<float4*>(out_f32 + row * ld_out + 4 * b) = make_float4(v[0], v[1], v[2], v[3]);
  if (out_bf16)
    *reinterpret_cast<uint2*>(out_bf16 + row * ld_out + 4 * b) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
}

__global__ void prepare_splits_kernel(const int32_t* __restrict__ splits, int32_t* __restrict__ quant,
                                      int32_t* __restrict__ merge, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t q = max(splits[i] - 1, 1);
  quant[i] = q;
  merge[i] = q + 1;
}

// Page table of the packed reader from SGLang's token -> slot map: one warp per (request,
// 64-token page).  Page p of request b is req_to_token[req[b]][64 p] / 64 when the page's
// tokens sit in 64 consecutive slots starting at a multiple of 64 (the packed pool hands out
// whole pages); otherwise the page is -1 and ROLAQ_DEV_BAD_PAGE is reported (the reader then
// skips it).  Pages past the request's length are -1.  The request lengths are copied to
// int32 alongside, the reader's seq_lens.
__global__ void page_table_kernel(const int32_t* __restrict__ req_to_token, int64_t rt_stride, const void* req_idx,
                                  int req64, const void* seq_lens, int seq64, int64_t batch, int32_t max_pages,
                                  int32_t* __restrict__ page_table, int64_t pt_stride, int32_t* __restrict__ seq_out,
                                  int32_t* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int p = blockIdx.x * (blockDim.x >> 5) + warp;
  if (b >= batch || p >= max_pages) return;
  const int64_t req = load_index(req_idx, req64, b);
  const int64_t L = load_index(seq_lens, seq64, b);
  if (p == 0 && lane == 0 && seq_out != nullptr) seq_out[b] = static_cast<int32_t>(L);
  int32_t page = -1;
  const int64_t t0 = static_cast<int64_t>(p) * 64;
  if (req >= 0 && t0 < L) {
    const int32_t* row = req_to_token + req * rt_stride + t0;
    const int32_t s0 = row[0];
    const int n = static_cast<int>(L - t0 < 64 ? L - t0 : 64);
    bool ok = s0 >= 0 && (s0 & 63) == 0;
    for (int j = lane; j < n; j += 32) ok = ok && row[j] == s0 + j;
    ok = __all_sync(0xFFFFFFFFu, ok);
    if (ok) {
      page = s0 >> 6;
    } else if (lane == 0) {
      report(err, ROLAQ_DEV_BAD_PAGE);
    }
  }
  if (lane == 0) page_table[b * pt_stride + p] = page;
}

static inline unsigned blocks_for(int64_t units, int threads) {
  return static_cast<unsigned>((units + threads - 1) / threads);
}

int launch_scatter_pack(const float* x, int64_t ldx, const void* slots, int slots64, int64_t n, int d,
                        rolaq_codec codec, uint8_t* codes, float* params, int64_t num_slots, int32_t* err,
                        cudaStream_t s) {
  if (n == 0) return ROLAQ_OK;
  scatter_pack_kernel<<<blocks_for(n * (d / 128), 128), 128, 0, s>>>(x, ldx, slots, slots64, n, d, codec, codes,
                                                                     params, num_slots, err);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

int launch_aux(const float* c, int64_t ldc, const uint16_t* k_pe, int64_t ld_pe, const int64_t* slots,
               const void* seq, int seq64, const void* req, int req64, const void* pos, int pos64, int64_t n,
               const rolaq_layer_cache& cache, int32_t* err, cudaStream_t s) {
  if (n == 0) return ROLAQ_OK;
  aux_kernel<<<blocks_for(n, 4), 128, 0, s>>>(c, ldc, k_pe, ld_pe, slots, seq, seq64, req, req64, pos, pos64, n,
                                              cache, err);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

int launch_dequant(const uint8_t* codes, const float* params, const void* slots, int slots64, int64_t n, int d,
                   int64_t num_slots, float* out_f32, uint16_t* out_bf16, int64_t ld_out, int32_t* err,
                   cudaStream_t s) {
  if (n == 0) return ROLAQ_OK;
  dequant_kernel<<<blocks_for(n * (d / 4), 256), 256, 0, s>>>(codes, params, slots, slots64, n, d, num_slots,
                                                              out_f32, out_bf16, ld_out, err);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

int launch_prepare_splits(const int32_t* splits, int32_t* quant, int32_t* merge, int64_t n, cudaStream_t s) {
  if (n == 0) return ROLAQ_OK;
  prepare_splits_kernel<<<blocks_for(n, 256), 256, 0, s>>>(splits, quant, merge, n);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

int launch_page_table(const int32_t* req_to_token, int64_t rt_stride, const void* req_idx, int req64,
                      const void* seq_lens, int seq64, int64_t batch, int32_t max_pages, int32_t* page_table,
                      int64_t pt_stride, int32_t* seq_out, int32_t* err, cudaStream_t s) {
  if (batch == 0 || max_pages == 0) return ROLAQ_OK;
  const dim3 grid(static_cast<unsigned>((max_pages + 7) / 8), static_cast<unsigned>(batch));
  page_table_kernel<<<grid, 256, 0, s>>>(req_to_token, rt_stride, req_idx, req64, seq_lens, seq64, batch, max_pages,
                                         page_table, pt_stride, seq_out, err);
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

}  // namespace rolaq
