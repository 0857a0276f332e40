// Fused packed-INT2 cache writer for sm_100a.
//
// c = c_kv @ R runs on tcgen05 tensor cores: each CTA keeps the R^T slice of one
// quantisation group resident in shared memory (loaded once by TMA, 128-byte swizzle) and
// streams c_kv rows through a 3-stage ring of two 64-wide K chunks each; one elected thread
// issues kind::f16 MMAs into one of four FP32 accumulators in tensor memory, and four sets
// of four epilogue warps (one warp per TMEM lane quarter) read the accumulators back
// (tcgen05.ld) to run the Lloyd INT2 codec, pack 4 codes per byte, scatter codes/params by
// slot, and write k_pe and the s4r16 window rows.  Set s takes every fourth tile of the CTA,
// so the codec of four tiles is in flight at once while the tensor core computes the next.
//
// Reference behaviour: deployment/sglang/QuantKernel/mla_fused_writer.py:54-224
// (FP32 GEMM + Triton _pack_and_aux) and mla_quant/oscar.py:120-144 (codec).
//
// CTA tile: 128 rows x 128 latent columns = one quantisation group.  CTA c serves group
// c % (D / 128) for every (#CTAs / groups)-th row tile, so the CTAs of one row tile run at
// the same time and the repeated reads of its rows hit L2.
#include "kernels.cuh"

namespace rolaq {

constexpr int kTileM = 128;
constexpr int kTileN = 128;  // one quantisation group
constexpr int kTileK = 64;   // one 128-byte swizzle row of BF16
constexpr int kStages = 3;
constexpr int kABytes = kTileM * kTileK * 2;  // 16 KB
constexpr int kBBytes = kTileN * kTileK * 2;  // 16 KB
constexpr int kStageBytes = 2 * kABytes;      // the ring streams c_kv only, two K chunks per stage
constexpr int kMaxKChunks = 8;                // D <= 512: the group's R^T slice (<= 128 KB) stays resident
constexpr int kNumBuf = 4;                       // TMEM accumulators = epilogue warp sets
constexpr int kEpiWarps = 4 * kNumBuf;           // one warp per TMEM lane quarter per set
constexpr int kWriterThreads = 32 * (2 + kEpiWarps);  // warp 0 TMA, warp 1 MMA, warps 2.. epilogue
constexpr int kSetThreads = 128;
constexpr uint32_t kTmemCols = kNumBuf * kTileN;  // 512
constexpr size_t kWriterSmem = size_t(kMaxKChunks) * kBBytes + size_t(kStages) * kStageBytes + 1024 + 256;

// Per-row bookkeeping shared by the codec epilogue warps of one row.
struct RowMeta {
  int64_t slot;
  int64_t ring;  // -1: not a window row
  bool ok;       // slot in range
};

// A row's slot check and ring row (window rules of the reference writer: sink positions and
// the last `recent` positions keep a BF16 copy in the request's ring), from its slot, seq
// length, request index and position (ignored when the call gives no positions: seq - 1).
__device__ __forceinline__ RowMeta row_meta_of(const WriterArgs& a, int64_t slot, int64_t seq, int64_t req,
                                               int64_t pos_or_neg1) {
  RowMeta m{0, -1, false};
  m.slot = slot;
  m.ok = slot >= 0 && slot < a.cache.num_slots;
  const int P = a.cache.sink, W = a.cache.recent;
  if (m.ok && slot > 0 && a.seq_lens != nullptr && a.req_idx != nullptr && a.cache.rows != nullptr &&
      (P + W) > 0) {
    const int64_t pos = a.positions ? pos_or_neg1 : seq - 1;
    const bool keep = (pos < P || pos >= seq - W) && req >= 0 && req < a.cache.max_reqs && pos >= 0;
    if (keep) {
      const int64_t w = W > 0 ? W : 1;
      const int64_t inner = pos < P ? pos : P + ((pos - P) > 0 ? (pos - P) : 0) % w;
      const int64_t ring = 1 + req * (P + W) + inner;
      m.ring = ring < a.cache.num_ring_rows ? ring : -1;
    }
  }
  return m;
}

__device__ __forceinline__ RowMeta row_meta(const WriterArgs& a, int64_t row, int64_t slot) {
  int64_t seq = 0, req = 0, pos = -1;
  if (slot > 0 && slot < a.cache.num_slots && a.seq_lens != nullptr && a.req_idx != nullptr &&
      a.cache.rows != nullptr) {
    seq = load_index(a.seq_lens, a.seq_is64, row);
    req = load_index(a.req_idx, a.req_is64, row);
    if (a.positions != nullptr) pos = load_index(a.positions, a.pos_is64, row);
  }
  return row_meta_of(a, slot, seq, req, pos);
}

// FP32 set: -1 when a >= b, else 0 (one instruction).
__device__ __forceinline__ int set_ge(float a, float b) {
  int r;
  asm("set.ge.s32.f32 %0, %1, %2;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}

// The smallest FP32 x with RN(x - m) >= b.  RN(x - m) never decreases as x grows, so
// [RN(x - m) >= b] is [x >= X]; X lies within a few ulps of RN(b + m).  False when the walk
// does not settle (the caller then takes the per-element path).
__device__ __forceinline__ bool sub_bound(float b, float m, float* X) {
  float x = __fadd_rn(b, m);
  if (__fsub_rn(x, m) >= b) {
#pragma unroll 1
    for (int k = 0; k < 16; ++k) {
      const float p = f32_prev(x);
      if (!(__fsub_rn(p, m) >= b)) {
        *X = x;
        return true;
      }
      x = p;
    }
  } else {
#pragma unroll 1
    for (int k = 0; k < 16; ++k) {
      x = f32_next(x);
      if (__fsub_rn(x, m) >= b) {
        *X = x;
        return true;
      }
    }
  }
  return false;
}

// Codes of one (row, 128-group) from the IEEE quotient per element: the reference's
// definition, used when the per-group bounds do not apply.  Warp-collective (TMEM loads);
// kept out of line so that the common path stays small.
__device__ __noinline__ void exact_code_words(uint32_t taddr, float mean, float stdv, float thr, uint32_t* words) {
  uint32_t r[32];
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    tmem_ld32(taddr + c * 32, r);
    tmem_wait_ld();
    reg_fence(r);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const uint32_t code = lloyd_code(__fsub_rn(__uint_as_float(r[j]), mean), stdv, thr);
      if (j < 16)
        w0 |= code << (2 * j);
      else
        w1 |= code << (2 * (j - 16));
    }
    words[2 * c] = w0;
    words[2 * c + 1] = w1;
  }
}

// Uniform min/max codes of one (row, group) (ROLAQ_CODEC_UNIFORM, OSCAR's baseline codec):
// the group's FP32 minimum and maximum, then one IEEE quotient per element.  Warp-collective
// (TMEM loads); its own instantiation of the kernel, so the learned-codec path is unchanged.
__device__ __forceinline__ void uniform_code_words(uint32_t taddr, uint32_t* words, float* scale_out,
                                                float* zero_out) {
  uint32_t r[32];
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    tmem_ld32(taddr + c * 32, r);
    tmem_wait_ld();
    reg_fence(r);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      mn = fminf(mn, __uint_as_float(r[j]));
      mx = fmaxf(mx, __uint_as_float(r[j]));
    }
  }
  const float scale = uniform_scale(mn, mx);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    tmem_ld32(taddr + c * 32, r);
    tmem_wait_ld();
    reg_fence(r);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const uint32_t code = uniform_code(__uint_as_float(r[j]), mn, scale);
      if (j < 16)
        w0 |= code << (2 * j);
      else
        w1 |= code << (2 * (j - 16));
    }
    words[2 * c] = w0;
    words[2 * c + 1] = w1;
  }
  *scale_out = scale;
  *zero_out = uniform_zero(mn, scale);
}

// The epilogue of one (row, group) of an accumulator: the thread's TMEM lane holds the row's
// 128 rotated values of the group at columns taddr .. taddr + 127.  kPlain: the rotated row
// (FP32 and / or BF16).  Otherwise the codec (mean, population variance, Lloyd codes from
// exact bounds), the packed codes and (scale, zero) by slot, the group's share of the k_pe
// copy, once per row (group 0) the slot <-> ring maps; window rows also go to the BF16 ring.
template <bool kPlain, bool kUniform>
__device__ __forceinline__ void epilogue_row_group(const WriterArgs& args, uint32_t taddr, int64_t row, bool valid,
                                                   int group, int d) {
  uint32_t r[32];

  if constexpr (kPlain) {
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      reg_fence(r);
      if (valid) {
        const int64_t col = group * 128 + c * 32;
        if (args.out_f32) {
          float4* dst = reinterpret_cast<float4*>(args.out_f32 + row * args.ld_out + col);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
        if (args.out_bf16) {
          uint4* dst = reinterpret_cast<uint4*>(args.out_bf16 + row * args.ld_out + col);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * j]), __uint_as_float(r[8 * j + 1])),
                                pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3])),
                                pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5])),
                                pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7])));
        }
      }
    }
  } else {
    uint32_t words[8];
    float scale, zero;
    if constexpr (kUniform) {
      uniform_code_words(taddr, words, &scale, &zero);
    } else {
    // pass 1: mean
    GroupSum acc;
    acc.zero();
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      reg_fence(r);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc.add(j & 7, __uint_as_float(r[j]));
    }
    const float mean = __fmul_rn(acc.total(), 1.0f / 128.0f);
    // pass 2: population variance of the centred values
    acc.zero();
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      reg_fence(r);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float df = __fsub_rn(__uint_as_float(r[j]), mean);
        acc.add(j & 7, __fmul_rn(df, df));
      }
    }
    const float var = __fmul_rn(acc.total(), 1.0f / 128.0f);
    const float stdv = __fsqrt_rn(__fadd_rn(var, 1e-8f));
    const float thr = args.codec.threshold;
    // pass 3: codes.  n = RN(diff / std) never decreases as diff grows, so each of the
    // reference's tests [n >= -t], [n >= 0], [n >= t] is diff >= an exact FP32 bound
    // found once per (row, group) (FP64 midpoint products; the middle one in closed
    // form), and diff = RN(x - mean) >= b is x >= X(b): three compares on the raw value
    // per element.  A std of 2^24 or more, or a search that does not settle, takes the
    // per-element quotient instead.
    float b_lo = 0.f, b_mid = 0.f, b_hi = 0.f;
    bool exact_all = !(stdv < 16777216.f);
    if (!exact_all) {
      b_mid = quotient_bound_zero(stdv);
      b_lo = quotient_bound(-thr, stdv);
      b_hi = quotient_bound(thr, stdv);
    }
    float x_lo = 0.f, x_mid = 0.f, x_hi = 0.f;
    if (!exact_all)
      exact_all = !(sub_bound(b_lo, mean, &x_lo) && sub_bound(b_mid, mean, &x_mid) &&
                    sub_bound(b_hi, mean, &x_hi));
    if (__any_sync(0xFFFFFFFFu, exact_all)) {
      exact_code_words(taddr, mean, stdv, thr, words);  // rare: the whole warp, quotient per element
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(taddr + c * 32, r);
        tmem_wait_ld();
        reg_fence(r);
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float x = __uint_as_float(r[j]);
          const int ncode = set_ge(x, x_lo) + set_ge(x, x_mid) + set_ge(x, x_hi);  // -code
          if (j < 16)
            w0 -= static_cast<uint32_t>(ncode) << (2 * j);
          else
            w1 -= static_cast<uint32_t>(ncode) << (2 * (j - 16));
        }
        words[2 * c] = w0;
        words[2 * c + 1] = w1;
      }
    }
    scale = __fmul_rn(args.codec.scale_factor, stdv);
    zero = __fsub_rn(args.codec.zero_const, __fdiv_rn(mean, scale));
    }
    RowMeta m{0, -1, false};
    if (valid) m = row_meta(args, row, args.slots[row]);
    if (valid && !m.ok && group == 0) report(args.err, ROLAQ_DEV_BAD_SLOT);
    if (valid && m.ok) {
      uint4* cdst = reinterpret_cast<uint4*>(args.cache.codes + m.slot * (d / 4) + group * 32);
      cdst[0] = make_uint4(words[0], words[1], words[2], words[3]);
      cdst[1] = make_uint4(words[4], words[5], words[6], words[7]);
      float2* pdst = reinterpret_cast<float2*>(args.cache.params + (m.slot * (d / 128) + group) * 2);
      *pdst = make_float2(scale, zero);
      if (args.k_pe != nullptr && m.slot > 0) {
        // k_pe: each group's epilogue copies its share of the row (all loads before the
        // stores), so that no group's CTAs carry the whole copy
        const int dr = args.cache.rope_dim, share = dr / (d / kTileN);
        const int j0 = (share % 8 == 0 && share <= 32) ? group * (share / 8) : (group == 0 ? 0 : dr / 8);
        const int j1 = (share % 8 == 0 && share <= 32) ? j0 + share / 8 : dr / 8;
        const uint4* src = reinterpret_cast<const uint4*>(args.k_pe + row * args.ld_pe);
        uint4* dst = reinterpret_cast<uint4*>(args.cache.rope + m.slot * dr);
        for (int j = j0; j < j1; j += 4) {
          uint4 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (j + u < j1) v[u] = src[j + u];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (j + u < j1) dst[j + u] = v[u];
        }
      }
      if (group == 0 && m.slot > 0) {
        // the slot <-> ring maps, once per row
        if (args.cache.rows != nullptr && args.seq_lens != nullptr && args.req_idx != nullptr) {
          args.cache.rows[m.slot] = static_cast<int32_t>(m.ring);
          if (m.ring >= 0) args.cache.owners[m.ring] = static_cast<int32_t>(m.slot);
        }
      }
    }
    // Window rows: BF16 rotated latent into the ring.  The TMEM loads are
    // warp-collective, so the whole warp reloads when any lane needs it.
    if (__any_sync(0xFFFFFFFFu, m.ring >= 0)) {
      uint4* hdst = m.ring >= 0 ? reinterpret_cast<uint4*>(args.cache.hp + m.ring * d + group * 128) : nullptr;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(taddr + c * 32, r);
        tmem_wait_ld();
        reg_fence(r);
        if (hdst != nullptr) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            hdst[c * 4 + j] =
                make_uint4(pack_bf16x2(__uint_as_float(r[8 * j]), __uint_as_float(r[8 * j + 1])),
                           pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3])),
                           pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5])),
                           pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7])));
        }
      }
    }
  }
}

// Issued before an epilogue waits for its accumulator: the row's slot, metadata and k_pe
// share into L2, so that the loads after the codec find them there.
template <bool kPlain>
__device__ __forceinline__ void epilogue_prefetch(const WriterArgs& args, int64_t row, int group, int d) {
  if constexpr (!kPlain) {
    if (row >= args.n) return;
    prefetch_line_l2(args.slots + row);
    if (args.seq_lens != nullptr)
      prefetch_line_l2(static_cast<const char*>(args.seq_lens) + row * (args.seq_is64 ? 8 : 4));
    if (args.req_idx != nullptr)
      prefetch_line_l2(static_cast<const char*>(args.req_idx) + row * (args.req_is64 ? 8 : 4));
    if (args.positions != nullptr)
      prefetch_line_l2(static_cast<const char*>(args.positions) + row * (args.pos_is64 ? 8 : 4));
    if (args.k_pe != nullptr)
      prefetch_line_l2(args.k_pe + row * args.ld_pe + group * (args.cache.rope_dim / (d / kTileN)));
  }
}

template <bool kPlain, bool kUniform = false>
__global__ void __launch_bounds__(kWriterThreads, 1)
    writer_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                  const WriterArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* bres = smem;                          // R^T slice of the CTA's group: kchunks x 16 KB
  uint8_t* ring = smem + kMaxKChunks * kBBytes;  // c_kv stages
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + kNumBuf;
  uint64_t* bfull = tempty + kNumBuf;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bfull + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int d = args.d;
  const int groups = d / kTileN;
  const int64_t row_tiles = (args.n + kTileM - 1) / kTileM;
  const int kchunks = d / kTileK;
  // One group per CTA (its R^T slice resident in shared memory): CTA c takes group c % groups
  // and the row tiles c / groups, + ctas_g, ...
  const int group = static_cast<int>(blockIdx.x % groups);
  const int64_t cg = blockIdx.x / groups;
  const int64_t ctas_g = (gridDim.x - group + groups - 1) / groups;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kNumBuf; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kSetThreads);
    }
    mbar_init(bfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_x);
    prefetch_tensormap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer -------------------------------------------------------------
    if (lane == 0) {
      mbar_expect_tx(bfull, static_cast<uint32_t>(kchunks * kBBytes));
      for (int kc = 0; kc < kchunks; ++kc)
        tma_load_2d(bres + kc * kBBytes, &tmap_w, bfull, kc * kTileK, group * kTileN);
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t rt = cg; rt < row_tiles; rt += ctas_g) {
        const int32_t row0 = static_cast<int32_t>(rt * kTileM);
        for (int kc = 0; kc < kchunks; kc += 2) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, args.err)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* a_s = ring + stage * kStageBytes;
          mbar_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(a_s, &tmap_x, &full[stage], kc * kTileK, row0);
          tma_load_2d(a_s + kABytes, &tmap_x, &full[stage], (kc + 1) * kTileK, row0);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (*(volatile int*)abort_flag) break;
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer -----------------------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t idesc = idesc_bf16(kTileM, kTileN);
      // Descriptors formed once: operands sit at fixed offsets from the ring and the resident
      // slice, and the 14-bit start-address field (addr >> 4) never carries within shared
      // memory, so each MMA's descriptors are the bases plus constants (two adds per MMA: the
      // issuing thread shares its sub-partition with epilogue warps).
      const uint64_t da0 = sw128_kmajor_desc(smem_u32(ring));
      const uint64_t db0 = sw128_kmajor_desc(smem_u32(bres));
      bool ok = mbar_wait(bfull, 0, args.err);
      int64_t lt = 0;
      for (int64_t rt = cg; ok && rt < row_tiles; rt += ctas_g, ++lt) {
        const int buf = static_cast<int>(lt % kNumBuf);
        const uint32_t use = static_cast<uint32_t>(lt / kNumBuf);
        if (!mbar_wait(&tempty[buf], (use & 1u) ^ 1u, args.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kTileN);
        for (int kc = 0; kc < kchunks; kc += 2) {
          if (!mbar_wait(&full[stage], phase, args.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = da0 + static_cast<uint64_t>((stage * kStageBytes) >> 4);
          const uint64_t db = db0 + static_cast<uint64_t>((kc * kBBytes) >> 4);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int k = 0; k < kTileK / 16; ++k) {
              umma_bf16_ss(d_tmem, da + static_cast<uint64_t>((h * kABytes + k * 32) >> 4),
                           db + static_cast<uint64_t>((h * kBBytes + k * 32) >> 4), idesc, (kc | h | k) != 0);
            }
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---- epilogue: set (w-2)/4 takes tiles lt = set, set + 4, ...; warp w reads TMEM lanes
    //      32*(w%4).. of accumulator lt % 4 -------------------------------------------------
    const int quad = warp & 3;
    const int set = (warp - 2) >> 2;
    int64_t lt = set;
    for (int64_t rt = cg + set * ctas_g; rt < row_tiles; rt += kNumBuf * ctas_g, lt += kNumBuf) {
      const int buf = static_cast<int>(lt % kNumBuf);
      const uint32_t use = static_cast<uint32_t>(lt / kNumBuf);
      const int64_t row = rt * kTileM + quad * 32 + lane;
      epilogue_prefetch<kPlain>(args, row, group, d);
      if (!mbar_wait(&tfull[buf], use & 1u, args.err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const bool valid = row < args.n;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * kTileN);
      epilogue_row_group<kPlain, kUniform>(args, taddr, row, valid, group, d);
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---- small batches (decode writes): SIMT rotation + codec -------------------------------
//
// For n <= kSmallWriteRows the tensor-core pipeline above is all fill and drain (one tile
// per group), so a CTA per (4 rows, group) computes its 4 x 128 rotated values with FP32
// FMAs (thread: one output column over one quarter of K in increasing k, its R^T loads all
// issued before the first FMA; the quarters added in order) and one warp per row runs the
// codec in the oracle's order: lane k < 8 keeps the
// running sum acc[k] over columns k, k + 8, .., and the tree
// ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)) is the xor-1, -2, -4 shuffle pairing.  The codes
// come from the same exact bounds as the tensor-core path; rolaq_rotate_rows takes the same
// path for the same n, so a batch's codes always match its own rotated values.
constexpr int kSmRows = 4;
constexpr int kSmThreads = 512;  // 128 output columns x 4 quarters of K
constexpr int64_t kSmallWriteRows = 256;

template <bool kPlain>
__global__ void __launch_bounds__(kSmThreads) small_writer_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                                                                  const uint16_t* __restrict__ w,
                                                                  const WriterArgs args) {
  __shared__ __align__(16) float xs[kSmRows][512];
  __shared__ float part[3][kSmRows][kTileN];
  __shared__ float cs[kSmRows][kTileN];
  const int d = args.d;
  const int group = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kSmRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Every independent global load is issued here, before any of them is used: this thread's
  // R^T quarter row, its 16-byte piece of the block's rows, and (lane 0 of warp r) row r's
  // slot and window metadata.
  const int col = tid & (kTileN - 1), quarter = tid >> 7, kq = d / 4;  // kq <= 128
  const uint16_t* wr = w + static_cast<int64_t>(group * kTileN + col) * d + quarter * kq;
  uint4 wv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (8 * i < kq) wv[i] = *reinterpret_cast<const uint4*>(wr + 8 * i);
  static_assert(kSmThreads >= kSmRows * 512 / 8, "one 16-byte piece of the rows per thread");
  const int xr = tid / (d / 8), xk8 = tid % (d / 8);
  uint4 xv = make_uint4(0, 0, 0, 0);
  if (xr < kSmRows && row0 + xr < args.n) xv = *reinterpret_cast<const uint4*>(x + (row0 + xr) * ldx + 8 * xk8);
  int64_t m_slot = 0, m_seq = 0, m_req = 0, m_pos = -1;
  if (!kPlain && warp < kSmRows && lane == 0 && row0 + warp < args.n) {
    const int64_t row = row0 + warp;
    m_slot = args.slots[row];
    if (args.seq_lens != nullptr) m_seq = load_index(args.seq_lens, args.seq_is64, row);
    if (args.req_idx != nullptr) m_req = load_index(args.req_idx, args.req_is64, row);
    if (args.positions != nullptr) m_pos = load_index(args.positions, args.pos_is64, row);
  }
  if (xr < kSmRows) {  // the block's rows as FP32
    const uint32_t ws[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      xs[xr][8 * xk8 + 2 * c] = bf16_lo(ws[c]);
      xs[xr][8 * xk8 + 2 * c + 1] = bf16_hi(ws[c]);
    }
  }
  __syncthreads();
  {
    float acc[kSmRows];
#pragma unroll
    for (int r = 0; r < kSmRows; ++r) acc[r] = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (8 * i >= kq) break;
      const float wf[8] = {bf16_lo(wv[i].x), bf16_hi(wv[i].x), bf16_lo(wv[i].y), bf16_hi(wv[i].y),
                           bf16_lo(wv[i].z), bf16_hi(wv[i].z), bf16_lo(wv[i].w), bf16_hi(wv[i].w)};
#pragma unroll
      for (int r = 0; r < kSmRows; ++r) {
        const float4 x0 = *reinterpret_cast<const float4*>(&xs[r][quarter * kq + 8 * i]);
        const float4 x1 = *reinterpret_cast<const float4*>(&xs[r][quarter * kq + 8 * i + 4]);
        acc[r] = fmaf(x0.x, wf[0], acc[r]);
        acc[r] = fmaf(x0.y, wf[1], acc[r]);
        acc[r] = fmaf(x0.z, wf[2], acc[r]);
        acc[r] = fmaf(x0.w, wf[3], acc[r]);
        acc[r] = fmaf(x1.x, wf[4], acc[r]);
        acc[r] = fmaf(x1.y, wf[5], acc[r]);
        acc[r] = fmaf(x1.z, wf[6], acc[r]);
        acc[r] = fmaf(x1.w, wf[7], acc[r]);
      }
    }
    if (quarter > 0) {
#pragma unroll
      for (int r = 0; r < kSmRows; ++r) part[quarter - 1][r][col] = acc[r];
    }
    __syncthreads();
    if (quarter == 0) {
#pragma unroll
      for (int r = 0; r < kSmRows; ++r)
        cs[r][col] = __fadd_rn(__fadd_rn(__fadd_rn(acc[r], part[0][r][col]), part[1][r][col]), part[2][r][col]);
    }
    __syncthreads();
  }
  if (warp >= kSmRows) return;
  const int64_t row = row0 + warp;
  if (row >= args.n) return;  // whole warp
  const float* c = cs[warp];
  const float4 v4 = *reinterpret_cast<const float4*>(c + 4 * lane);  // this lane's columns 4l .. 4l + 3
  const float v[4] = {v4.x, v4.y, v4.z, v4.w};
  if constexpr (kPlain) {
    const int64_t col = group * kTileN + 4 * lane;
    if (args.out_f32) *reinterpret_cast<float4*>(args.out_f32 + row * args.ld_out + col) = v4;
    if (args.out_bf16)
      *reinterpret_cast<uint2*>(args.out_bf16 + row * args.ld_out + col) =
          make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
    return;
  } else {
    // group sums in the fixed order (lanes 0..7 hold the running sums, the tree by shuffles)
    auto group_total = [&](auto term) {
      float a = 0.f;
      if (lane < 8) {
#pragma unroll
        for (int i = 0; i < kTileN / 8; ++i) a = __fadd_rn(a, term(c[8 * i + lane]));
      }
      const float t1 = __fadd_rn(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
      const float t2 = __fadd_rn(t1, __shfl_xor_sync(0xFFFFFFFFu, t1, 2));
      const float t3 = __fadd_rn(t2, __shfl_xor_sync(0xFFFFFFFFu, t2, 4));
      return __shfl_sync(0xFFFFFFFFu, t3, 0);
    };
    uint32_t byte = 0;
    float scale, zero;
    if (args.codec.family == ROLAQ_CODEC_UNIFORM) {  // min / max over the warp's 128 values
      float mn = fminf(fminf(v[0], v[1]), fminf(v[2], v[3])), mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
      }
      scale = uniform_scale(mn, mx);
      zero = uniform_zero(mn, scale);
#pragma unroll
      for (int q = 0; q < 4; ++q) byte |= uniform_code(v[q], mn, scale) << (2 * q);
    } else {
    const float mean = __fmul_rn(group_total([](float x) { return x; }), 1.0f / 128.0f);
    const float var = __fmul_rn(group_total([&](float x) {
                                  const float df = __fsub_rn(x, mean);
                                  return __fmul_rn(df, df);
                                }), 1.0f / 128.0f);
    const float stdv = __fsqrt_rn(__fadd_rn(var, 1e-8f));
    const float thr = args.codec.threshold;
    if (stdv < 16777216.f) {  // exact bounds: three compares per element
      const float b_lo = quotient_bound(-thr, stdv), b_mid = quotient_bound_zero(stdv),
                  b_hi = quotient_bound(thr, stdv);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float df = __fsub_rn(v[q], mean);
        byte |= (static_cast<uint32_t>(df >= b_lo) + static_cast<uint32_t>(df >= b_mid) +
                 static_cast<uint32_t>(df >= b_hi)) << (2 * q);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) byte |= lloyd_code(__fsub_rn(v[q], mean), stdv, thr) << (2 * q);
    }
    scale = __fmul_rn(args.codec.scale_factor, stdv);
    zero = __fsub_rn(args.codec.zero_const, __fdiv_rn(mean, scale));
    }
    const RowMeta m = row_meta_of(args, __shfl_sync(0xFFFFFFFFu, m_slot, 0), __shfl_sync(0xFFFFFFFFu, m_seq, 0),
                                  __shfl_sync(0xFFFFFFFFu, m_req, 0), __shfl_sync(0xFFFFFFFFu, m_pos, 0));
    if (!m.ok) {
      if (group == 0 && lane == 0) report(args.err, ROLAQ_DEV_BAD_SLOT);
      return;
    }
    args.cache.codes[m.slot * (d / 4) + group * 32 + lane] = static_cast<uint8_t>(byte);
    if (lane == 0)
      *reinterpret_cast<float2*>(args.cache.params + (m.slot * (d / 128) + group) * 2) = make_float2(scale, zero);
    if (group == 0 && m.slot > 0) {
      const int dr = args.cache.rope_dim;
      if (args.k_pe != nullptr && lane < dr / 8)
        reinterpret_cast<uint4*>(args.cache.rope + m.slot * dr)[lane] =
            reinterpret_cast<const uint4*>(args.k_pe + row * args.ld_pe)[lane];
      if (lane == 0 && args.cache.rows != nullptr && args.seq_lens != nullptr && args.req_idx != nullptr) {
        args.cache.rows[m.slot] = static_cast<int32_t>(m.ring);
        if (m.ring >= 0) args.cache.owners[m.ring] = static_cast<int32_t>(m.slot);
      }
    }
    if (m.ring >= 0)  // window row: the BF16 rotated latent into the ring
      *reinterpret_cast<uint2*>(args.cache.hp + m.ring * d + group * kTileN + 4 * lane) =
          make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  }
}

// ---- host side -----------------------------------------------------------------------

// 2-D BF16 (or byte) tensor map over a row-major matrix, 128-byte swizzle.
int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ROLAQ_ECUDA;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ROLAQ_OK : ROLAQ_ECUDA;
}

int launch_writer(const uint16_t* x, int64_t ldx, const uint16_t* w, const WriterArgs& args, bool plain,
                  cudaStream_t stream) {
  CUtensorMap mx, mw;
  const int d = args.d;
  if (args.n <= 0) return ROLAQ_OK;
  if (d % (2 * kTileK) != 0 || d / kTileK > kMaxKChunks) return ROLAQ_EUNSUPPORTED;
  if (args.n <= kSmallWriteRows) {
    const dim3 grid(static_cast<unsigned>((args.n + kSmRows - 1) / kSmRows), static_cast<unsigned>(d / kTileN));
    if (plain)
      small_writer_kernel<true><<<grid, kSmThreads, 0, stream>>>(x, ldx, w, args);
    else
      small_writer_kernel<false><<<grid, kSmThreads, 0, stream>>>(x, ldx, w, args);
    return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
  }
  int rc = make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<uint64_t>(d),
                       static_cast<uint64_t>(args.n), static_cast<uint64_t>(ldx) * 2, kTileK, kTileM);
  if (rc != ROLAQ_OK) return rc;
  rc = make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<uint64_t>(d), static_cast<uint64_t>(d),
                   static_cast<uint64_t>(d) * 2, kTileK, kTileN);
  if (rc != ROLAQ_OK) return rc;
  const int groups = d / kTileN;
  const int64_t tiles = ((args.n + kTileM - 1) / kTileM) * groups;
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  // The attribute is set once per process (and per kernel), not on every launch, so
  // that launches can be captured into CUDA graphs without extra API calls.
  static const bool attr_plain =
      cudaFuncSetAttribute(writer_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kWriterSmem) ==
      cudaSuccess;
  static const bool attr_codec =
      cudaFuncSetAttribute(writer_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kWriterSmem) ==
      cudaSuccess;
  static const bool attr_uniform =
      cudaFuncSetAttribute(writer_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kWriterSmem) == cudaSuccess;
  const bool uniform = !plain && args.codec.family == ROLAQ_CODEC_UNIFORM;
  if (!(plain ? attr_plain : (uniform ? attr_uniform : attr_codec))) return ROLAQ_ECUDA;
  if (plain) {
    writer_kernel<true><<<grid, kWriterThreads, kWriterSmem, stream>>>(mx, mw, args);
  } else if (uniform) {
    writer_kernel<false, true><<<grid, kWriterThreads, kWriterSmem, stream>>>(mx, mw, args);
  } else {
    writer_kernel<false><<<grid, kWriterThreads, kWriterSmem, stream>>>(mx, mw, args);
  }
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

}  // namespace rolaq
