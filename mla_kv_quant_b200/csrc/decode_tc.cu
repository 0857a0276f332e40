// Packed-INT2 MLA decode attention on tcgen05 tensor cores (sm_100a), one kernel template
// over (D, Dr, H): DeepSeek-V2-Lite / Moonlight (512, 64, 16), MiniCPM3 (256, 32, 40), and
// (512, 64, 8), (256, 32, 16).
//
// Reference behaviour: upstream packed_mla_decode_gf_fwd called at
// deployment/patches/rolaq_sglang.patch:51-111; queries in the rotated frame
// (deployment/sglang/srt/mem_cache/rolaq_mla.py:56-71).
//
// One CTA per (request, KV split) walks its split in tiles of 128 tokens (two 64-slot
// pages).  The dequantised latent of token t in group g is s_tg (c_te - z_tg); the
// kernel never forms it:
//   q . c_hat = sum_g s_g (q_g . c - z_g sum(q_g))          (scores)
//   sum_t P_t c_hat_t = sum_g [sum_t (P_t s_tg) c_t - sum_t (P_t s_tg) z_tg]   (PV)
// Codes enter the tensor cores as FP8 E4M3 bytes holding c or 4c: the E4M3 patterns
// 0..15 are exactly p * 2^-9 (subnormals continue linearly into the first normal
// binade), so `w & 0x03030303` and `w & 0x0C0C0C0C` turn a packed word into four
// exact operands with one AND each.  Elements stored as 4c get a query weight of 1/4
// (QK) and an output weight of 1/4 (PV).
//
// Per tile:
//   * 16 token warps, four threads per token (thread k: a quarter of the token's code
//     bytes, the softmax of the head set k = heads [H/4 k, H/4 (k+1))) expand the codes
//     into TMEM (A of QK^T, lane = token) and into an MN-major smem tile (A of PV, row =
//     token);
//   * QK^T = kind::f8f6f4, M = 128 tokens, N = 2H (per head a hi and a lo E4M3 term of
//     the query, exact for BF16 after a per-head power-of-two scale), + the rope part in
//     kind::f16 with k_pe staged by TMA;
//   * the token threads turn scores into P = 2^(s - m_ref) against a reference max that
//     moves only when a tile max exceeds it by more than kTau (lazy rescaling; the tile
//     maxima are exchanged among the four warps of a head set, 128 threads), and
//     write P' = P s_g E_g (E_g a per-group power of two that moves only when the group
//     scale outgrows it) as two E4M3 terms;
//   * PV = kind::f8f6f4 (M = 128 latent elements of a group, N = 2H, K = 128 tokens)
//     accumulates straight into a TMEM O accumulator across all tiles.
// When m_ref or E_g moves, each token warp rescales the O columns of its own heads in
// TMEM (lane quarter = its tokens' quarter) and, at the end, writes those columns.  An MMA
// warp issues QK^T(i+1) as soon as its codes are in TMEM and PV(i) as soon as P'(i) is in
// shared memory; a producer warp keeps the k_pe TMA, the params bulk copies and the L2
// prefetch ahead; all three roles are driven by mbarriers.
#include "kernels.cuh"

namespace rolaq {
namespace tc {

constexpr int TILE = 128, PAGE = 64;
// 16 token warps + an MMA warp + a producer warp (18 warps: at most 5 per SM sub-partition
// -> 96 registers); the MMA and producer warps sit on different sub-partitions.
constexpr int NTOK_WARPS = 16;
constexpr int TOK_THREADS = NTOK_WARPS * 32;
constexpr int MMA_WARP = NTOK_WARPS;
constexpr int THREADS = TOK_THREADS + 64;
// P' = 2^(s - m_ref) s_g E_g < 2^kTau * kEMax = 362 stays inside E4M3 (448).
constexpr float kTau = 4.5f;    // m_ref moves when a tile max exceeds it by more than this (log2 units)
constexpr float kEMax = 16.f;   // E_g moves when max_t s_tg * E_g reaches this (set to [4, 8))
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
static_assert(kEMax * 22.7f < 448.f, "P' must stay below the largest E4M3 value");

template <int D_, int DR_, int H_>
struct Cfg {
  static constexpr int D = D_, DR = DR_, H = H_;
  static constexpr int NG = D / 128;               // quantisation groups per token
  static constexpr int HS = H / 4;                 // heads per head set
  static constexpr int NQ = 2 * H;                 // N of QK^T and PV: a hi and a lo term per head
  static constexpr int NPE = (H + 15) / 16 * 16;   // N of the rope MMA (rows >= H are zero)
  static constexpr int EW = D / 16;                // code bytes (= expanded FP8 words) per token thread
  static constexpr int SLOTS = HS + NG;            // decision state per head set, one per lane
  static constexpr int SLOT_PAD = (SLOTS + 3) / 4 * 4;
  static constexpr int PB_ROW = NQ <= 32 ? 32 : 128;  // bytes per token row of a P' tile (SW32 / SW128)
  static_assert(H % 8 == 0 && HS % 2 == 0 && NQ <= 256 && SLOTS <= 16, "head layout");
  static_assert((D == 512 || D == 256) && (DR == 64 || DR == 32), "latent / rope widths");
  // ---- shared memory (offsets from a 1024-byte aligned base) ----
  static constexpr int KPE_STAGE = TILE * DR * 2;  // k_pe of the tile, K-major SW128 / SW64 (TMA)
  static constexpr int PVA_GROUP = TILE * 128;     // 128 tokens x 128 B, MN-major SW128
  static constexpr int PVA_BUF = NG * PVA_GROUP;
  static constexpr int QB_GROUP = NQ * 128;        // NQ query rows x 128 B, K-major SW128
  static constexpr int QPE_BYTES = NPE * DR * 2;   // NPE rows of q_pe, K-major SW128 / SW64
  static constexpr int PB_GROUP = TILE * PB_ROW;   // 128 tokens x PB_ROW B, MN-major
  static constexpr int PB_BUF = NG * PB_GROUP;
  static constexpr int PAR_STAGE = TILE * NG * 2 * 4;  // (scale, zero) x NG per token (bulk copy)
  static constexpr int OFF_KPE = 0;
  static constexpr int OFF_PVA = OFF_KPE + 2 * KPE_STAGE;
  static constexpr int OFF_QB = OFF_PVA + 2 * PVA_BUF;
  static constexpr int OFF_QPE = OFF_QB + NG * QB_GROUP;
  static constexpr int OFF_PB = (OFF_QPE + QPE_BYTES + 1023) / 1024 * 1024;
  static constexpr int OFF_PAR = OFF_PB + 2 * PB_BUF;
  static constexpr int OFF_F = OFF_PAR + 2 * PAR_STAGE;
  // float scratch
  static constexpr int F_QSUM = 0;                          // [NG][H]   sum of the query over the group
  static constexpr int F_KINV = F_QSUM + NG * H;            // [H]       2^(9 - k_h)
  static constexpr int F_TAB = (F_KINV + H + 3) / 4 * 4;    // [2][4][4][SLOT_PAD] tile maxima per head set,
                                                            //           token quarter, slot (heads, groups)
  static constexpr int F_FINL = F_TAB + 2 * 4 * 4 * SLOT_PAD;  // [H][4]      sum P per head and token quarter
  static constexpr int F_FINY = F_FINL + 4 * H;                // [NG][H][4]  sum P' z per group, head, quarter
  static constexpr int F_TOTAL = F_FINY + 4 * NG * H;
  static constexpr int OFF_BAR = OFF_F + ((F_TOTAL * 4 + 15) / 16) * 16;
  static constexpr int OFF_TMEMSLOT = OFF_BAR + 12 * 8;
  static constexpr size_t SMEM = size_t(OFF_TMEMSLOT) + 16 + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(OFF_PVA % 1024 == 0 && OFF_QB % 1024 == 0 && OFF_QPE % 1024 == 0 && OFF_PB % 1024 == 0 &&
                    QB_GROUP % 1024 == 0 && OFF_PAR % 16 == 0,
                "swizzle-atom alignment of the operand tiles");
  // ---- TMEM columns (every MMA accumulator starts at a multiple of 32 columns) ----
  static constexpr int GSC = (NQ + 31) / 32 * 32;      // columns per group block of QK^T and O
  static constexpr uint32_t T_AQK = 0;                 // D/4 cols: FP8 codes of the tile (lane = token)
  static constexpr uint32_t T_DQK = D / 4;             // NG blocks of NQ cols: QK^T, [set k: hi HS, lo HS]
  static constexpr uint32_t T_DPE = T_DQK + NG * GSC;  // NPE cols: rope scores
  static constexpr uint32_t T_O = (T_DPE + NPE + 31) / 32 * 32;  // NG blocks: O, same column order
  static_assert(T_O + NG * GSC <= 512, "TMEM columns");
  // column alignment of the per-thread TMEM accesses (start = base + stride * k)
  static constexpr int AL_Q = pow2_align(2 * HS);  // QK^T and O columns of head set k
  static constexpr int AL_P = pow2_align(HS);      // rope columns of head set k
  static constexpr int AL_A = pow2_align(EW);      // code columns of thread k
};
// barriers
// B_KFREE[s]: QK^T of the tile in k_pe stage s has completed (producer may refill it);
// B_PFREE[s]: the token threads have read params stage s.  Per-stage barriers keep every
// waiter within one phase of the barrier it waits on.
constexpr int B_KPE = 0, B_QK = 2, B_PV = 3, B_AQK = 4, B_PREADY = 5, B_PAR = 6, B_KFREE = 8, B_PFREE = 10;

__device__ __forceinline__ uint32_t sw128(int row, int byte) {  // 128-byte rows, 1024-byte atoms
  return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + (((byte >> 4) ^ (row & 7)) << 4) +
                               (byte & 15));
}
__device__ __forceinline__ uint32_t sw64(int row, int byte) {  // 64-byte rows, 512-byte atoms
  return static_cast<uint32_t>((row >> 3) * 512 + (row & 7) * 64 + (((byte >> 4) ^ ((row >> 1) & 3)) << 4) +
                               (byte & 15));
}
__device__ __forceinline__ uint32_t sw32(int row, int byte) {  // 32-byte rows, 256-byte atoms
  return static_cast<uint32_t>((row >> 3) * 256 + (row & 7) * 32 + (((byte >> 4) ^ ((row >> 2) & 1)) << 4) +
                               (byte & 15));
}

__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// E_g for a tile whose largest group scale is gm >= 0: the power of two with gm * E in [4, 8).
__device__ __forceinline__ float group_e(float gm) {
  int eb = (__float_as_int(gm) >> 23) & 0xFF;
  eb = min(max(eb, 29), 225);
  return __int_as_float((256 - eb) << 23);
}

// a / b for powers of two a <= b in the normal range (exact by exponent arithmetic; a ratio
// below 2^-126 becomes 2^-126, which only arises when the accumulator it scales is empty).
__device__ __forceinline__ float pow2_ratio(float a, float b) {
  return __int_as_float(max(__float_as_int(a) - __float_as_int(b) + (127 << 23), 1 << 23));
}

// K index (position in a row of FP8 operand bytes) <-> element of the group; an involution.
__device__ __forceinline__ int kperm(int w) { return (w & ~15) | ((w & 3) << 2) | ((w >> 2) & 3); }

// Four FP8 operand words per packed code word: byte b of out[j] is element 4b + j of the
// word's 16 codes (c for even j, 4c for odd j).
__device__ __forceinline__ void expand_word(uint32_t w, uint32_t* out) {
  const uint32_t w4 = w >> 4;
  out[0] = w & 0x03030303u;   // c of element 4b + 0, byte b
  out[1] = w & 0x0C0C0C0Cu;   // 4c of element 4b + 1
  out[2] = w4 & 0x03030303u;  // c of element 4b + 2
  out[3] = w4 & 0x0C0C0C0Cu;  // 4c of element 4b + 3
}

// Sum of v over the 32 lanes of a warp (every lane gets it).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

template <int D, int DR, int H>
__global__ void __launch_bounds__(THREADS, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tm_rope, const DecodeArgs a) {
  using C = Cfg<D, DR, H>;
  constexpr int NG = C::NG, HS = C::HS, NQ = C::NQ, EW = C::EW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* F = reinterpret_cast<float*>(smem + C::OFF_F);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEMSLOT);

  const int b = blockIdx.y, split = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the window/merge kernel that follows may start its window phase on SMs this grid frees
  if (tid == 0) grid_launch_dependents();
  const int S = a.num_splits + 1;  // the window split (index num_splits) is written by another kernel
  int L = a.seq_lens[b];
  if (L < 0) L = 0;
  if (L > a.max_pages * PAGE) {
    if (tid == 0) report(a.err, ROLAQ_DEV_BAD_REQ);
    L = a.max_pages * PAGE;
  }
  const int P = a.cache.sink, W = a.cache.recent;
  int lo = min(P, L);
  int hi = max(lo, L - W);
  if (a.token_range != nullptr) {
    lo = max(lo, a.token_range[2 * b]);
    hi = max(lo, min(hi, a.token_range[2 * b + 1]));
  }
  const int first_page = lo / PAGE;
  const int npages = hi > lo ? (hi - 1) / PAGE - first_page + 1 : 0;
  // The range's 128-token tiles (page pairs) spread over the splits as evenly as they go:
  // the first (tiles % num_splits) splits take one tile more.
  const int all_tiles = (npages + 1) / 2;
  const int tbase = all_tiles / a.num_splits, textra = all_tiles % a.num_splits;
  const int p0 = first_page + 2 * (split * tbase + min(split, textra));
  const int p1 = min(first_page + npages, p0 + 2 * (tbase + (split < textra ? 1 : 0)));
  if (p0 >= p1) {
    for (int u = tid; u < H * D; u += blockDim.x) {
      const int h = u / D, j = u % D;
      a.part_o[((static_cast<int64_t>(b) * H + h) * S + split) * D + j] = 0.f;
    }
    if (tid < H) a.part_lse[(static_cast<int64_t>(b) * H + tid) * S + split] = -INFINITY;
    return;
  }
  const int ntiles = (p1 - p0 + 1) / 2;

  // Page ids are fetched ahead of use (page_raw: an unconditional load from a clamped
  // index, so that nothing waits on it until it is used) and checked when used
  // (page_of: absence is a property of the tile index, not of the loaded value).
  auto page_raw = [&](int i, int half) -> int32_t {
    return a.page_table[b * a.pt_stride + min(p0 + 2 * i + half, p1 - 1)];
  };
  auto page_of = [&](int i, int half, int32_t raw) -> int64_t {  // pool page; -1 absent, -2 out of range
    if (p0 + 2 * i + half >= p1) return -1;
    return (raw >= 0 && (static_cast<int64_t>(raw) + 1) * PAGE <= a.cache.num_slots) ? raw : -2;
  };
  // k_pe of tile i (page ids r0, r1) into stage i & 1 (elected thread)
  auto issue_kpe = [&](int i, int32_t r0, int32_t r1) {
    const int s = i & 1;
    const int64_t pg0 = page_of(i, 0, r0), pg1 = page_of(i, 1, r1);
    const uint32_t bytes = (pg0 >= 0 ? PAGE * DR * 2 : 0) + (pg1 >= 0 ? PAGE * DR * 2 : 0);
    if (pg0 == -2 || pg1 == -2) report(a.err, ROLAQ_DEV_BAD_PAGE);
    if (bytes == 0) {
      mbar_arrive(&bars[B_KPE + s]);
      return;
    }
    mbar_expect_tx(&bars[B_KPE + s], bytes);
    uint8_t* st = smem + C::OFF_KPE + s * C::KPE_STAGE;
    if (pg0 >= 0) tma_load_2d(st, &tm_rope, &bars[B_KPE + s], 0, static_cast<int32_t>(pg0 * PAGE));
    if (pg1 >= 0)
      tma_load_2d(st + PAGE * DR * 2, &tm_rope, &bars[B_KPE + s], 0, static_cast<int32_t>(pg1 * PAGE));
  };
  // (scale, zero) rows of tile i into params stage i & 1 (elected thread)
  auto issue_params = [&](int i, int32_t r0, int32_t r1) {
    const int s = i & 1;
    const int64_t pg0 = page_of(i, 0, r0), pg1 = page_of(i, 1, r1);
    const uint32_t bytes = (pg0 >= 0 ? C::PAR_STAGE / 2 : 0) + (pg1 >= 0 ? C::PAR_STAGE / 2 : 0);
    if (bytes == 0) {
      mbar_arrive(&bars[B_PAR + s]);
      return;
    }
    mbar_expect_tx(&bars[B_PAR + s], bytes);
    uint8_t* st = smem + C::OFF_PAR + s * C::PAR_STAGE;
    if (pg0 >= 0) bulk_load(st, a.cache.params + pg0 * PAGE * NG * 2, C::PAR_STAGE / 2, &bars[B_PAR + s]);
    if (pg1 >= 0)
      bulk_load(st + C::PAR_STAGE / 2, a.cache.params + pg1 * PAGE * NG * 2, C::PAR_STAGE / 2, &bars[B_PAR + s]);
  };
  auto prefetch_tile = [&](int i, int32_t r0, int32_t r1) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int64_t pg = page_of(i, half, half ? r1 : r0);
      if (pg < 0) continue;
      prefetch_l2(a.cache.codes + pg * PAGE * (D / 4), PAGE * (D / 4));
      prefetch_l2(a.cache.params + pg * PAGE * NG * 2, PAGE * NG * 2 * 4);
      prefetch_l2(a.cache.rope + pg * PAGE * DR, PAGE * DR * 2);
    }
  };

  // token threads: the page ids of tiles 0 and 1, loaded before the set-up (their latency
  // overlaps the query preparation)
  int32_t raw0 = 0, raw1 = 0;
  if (warp < NTOK_WARPS) {
    raw0 = page_raw(0, (32 * (warp & 3) + lane) >> 6);
    raw1 = page_raw(1, (32 * (warp & 3) + lane) >> 6);
  }
  // ---- set-up ---------------------------------------------------------------------------
  if (tid == 0) {
    mbar_init(&bars[B_KPE], 1);
    mbar_init(&bars[B_KPE + 1], 1);
    mbar_init(&bars[B_PAR], 1);
    mbar_init(&bars[B_PAR + 1], 1);
    mbar_init(&bars[B_QK], 1);
    mbar_init(&bars[B_PV], 1);
    mbar_init(&bars[B_AQK], TOK_THREADS);
    mbar_init(&bars[B_PREADY], TOK_THREADS);
    for (int st = 0; st < 2; ++st) {
      mbar_init(&bars[B_KFREE + st], 1);
      mbar_init(&bars[B_PFREE + st], TOK_THREADS);
    }
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // queries: per-head scale 2^k_h, E4M3 hi/lo B tiles in the K order of the code bytes
  // (odd elements weighted 1/4), group sums, rope rows.  A head's D elements are D/16 parts
  // of 16, one lane each; a warp takes 32 / (D/16) heads per round.
  if (tid < TOK_THREADS) {
    constexpr int PPH = D / 16;        // lanes (parts) per head
    constexpr int HPW = 32 / PPH;      // heads per warp per round
    constexpr int ROUNDS = (H + NTOK_WARPS * HPW - 1) / (NTOK_WARPS * HPW);
    // zero q_pe rows past the last head (their N columns of the rope MMA are never read)
    for (int u = tid; u < (C::NPE - H) * DR / 8; u += TOK_THREADS)
      *reinterpret_cast<uint4*>(smem + C::OFF_QPE + (H * DR / 8 + u) * 16) = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int rd = 0; rd < ROUNDS; ++rd) {
      const int h = (rd * NTOK_WARPS + warp) * HPW + lane / PPH, part = lane % PPH;  // elements [16 part, +16)
      const bool valid = h < H;
      const uint16_t* qh = a.q + b * a.q_sb + min(h, H - 1) * a.q_sh;
      float v[16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(qh + 16 * part + 8 * c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[8 * c + 2 * k] = bf16_lo(ws[k]);
          v[8 * c + 2 * k + 1] = bf16_hi(ws[k]);
        }
      }
      float mx = 0.f, sum = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        mx = fmaxf(mx, fabsf(v[e]));
        sum += v[e];
      }
#pragma unroll
      for (int o = PPH / 2; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
#pragma unroll
      for (int o = 1; o <= 4; o <<= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);  // 8 parts per group
      int ex = 0;
      if (mx > 0.f) frexpf(mx, &ex);  // mx < 2^ex
      ex = min(max(ex, -100), 100);
      const int kh = 7 - ex;  // |q| * 2^kh < 128
      const float qs = pow2i(kh);
      if (!valid) continue;
      if (part == 0) F[C::F_KINV + h] = pow2i(9 - kh);
      const int g = part >> 3;
      if ((part & 7) == 0) F[C::F_QSUM + g * H + h] = sum;
      uint8_t* qb = smem + C::OFF_QB + g * C::QB_GROUP;
      const int row_hi = 2 * HS * (h / HS) + (h % HS), row_lo = row_hi + HS;
      // The 16 elements fill one 16-byte chunk of each row in the K order of the code bytes:
      // byte j holds element kperm(j) = 4 (j & 3) + (j >> 2), so word w holds elements w, w + 4,
      // w + 8, w + 12 (all of w's parity, hence one weight).
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float sw = qs * ((w & 1) ? 0.25f : 1.f);
        const float x0 = v[w] * sw, x1 = v[w + 4] * sw, x2 = v[w + 8] * sw, x3 = v[w + 12] * sw;
        const uint32_t h01 = f32x2_to_e4m3x2(x0, x1), h23 = f32x2_to_e4m3x2(x2, x3);
        const __half2 f01 = e4m3x2_to_half2(h01), f23 = e4m3x2_to_half2(h23);
        const uint32_t l01 = f32x2_to_e4m3x2((x0 - __low2float(f01)) * 16.f, (x1 - __high2float(f01)) * 16.f);
        const uint32_t l23 = f32x2_to_e4m3x2((x2 - __low2float(f23)) * 16.f, (x3 - __high2float(f23)) * 16.f);
        hw[w] = __byte_perm(h01, h23, 0x5410);
        lw[w] = __byte_perm(l01, l23, 0x5410);
      }
      *reinterpret_cast<uint4*>(qb + sw128(row_hi, 16 * (part & 7))) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(qb + sw128(row_lo, 16 * (part & 7))) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      if (part < DR / 8) {  // rope part of the query: BF16 row of DR into a K-major swizzled tile
        const uint4 w = *reinterpret_cast<const uint4*>(qh + D + 8 * part);
        const uint32_t off = DR == 64 ? sw128(h, 16 * part) : sw64(h, 16 * part);
        *reinterpret_cast<uint4*>(smem + C::OFF_QPE + off) = w;
      }
    }
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool alive = true;
  const uint32_t id_qk = idesc_e4m3(128, NQ, 0, 0);
  const uint32_t id_pe = idesc_bf16(128, C::NPE);
  const uint32_t id_pv = idesc_e4m3(128, NQ, 1, 1);
  // Descriptors: a tile's operands sit at fixed offsets from a few bases; within 227 KB the
  // start-address field (addr >> 4, 14 bits) never carries, so offsets are plain adds.
  auto issue_qk = [&](int i, uint64_t dq0, uint64_t dk0, uint64_t dqp) {
#pragma unroll
    for (int g = 0; g < NG; ++g) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f8_ts(tmem + C::T_DQK + C::GSC * g, tmem + C::T_AQK + 32 * g + 8 * kk,
                   dq0 + static_cast<uint64_t>((C::QB_GROUP >> 4) * g + 2 * kk), id_qk, kk > 0);
    }
    const uint64_t dk = dk0 + static_cast<uint64_t>((i & 1) * (C::KPE_STAGE >> 4));
#pragma unroll
    for (int kk = 0; kk < DR / 16; ++kk) umma_bf16_ss(tmem + C::T_DPE, dk + 2 * kk, dqp + 2 * kk, id_pe, kk > 0);
    umma_commit(&bars[B_QK]);
    umma_commit(&bars[B_KFREE + (i & 1)]);
  };
  auto issue_pv = [&](int i, uint64_t dpa0, uint64_t dpb0) {
    const uint64_t da = dpa0 + static_cast<uint64_t>((i & 1) * (C::PVA_BUF >> 4));
    const uint64_t db = dpb0 + static_cast<uint64_t>((i & 1) * (C::PB_BUF >> 4));
#pragma unroll
    for (int g = 0; g < NG; ++g) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f8_ss(tmem + C::T_O + C::GSC * g, da + static_cast<uint64_t>((C::PVA_GROUP >> 4) * g + 256 * kk),
                   db + static_cast<uint64_t>((C::PB_GROUP >> 4) * g + (32 * C::PB_ROW >> 4) * kk), id_pv,
                   (i > 0 || kk > 0) ? 1u : 0u);
    }
    umma_commit(&bars[B_PV]);
  };

  if (warp < NTOK_WARPS) {
    // ---- token warps ------------------------------------------------------------------------
    const int q4 = warp & 3, k = warp >> 2;
    const int t = 32 * q4 + lane;  // token of the tile (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(32 * q4) << 16;
    const float sl2 = a.sm_scale * kLog2e;
    // this thread's code bytes: [EW k, EW (k + 1)) of the token's row = group kg, bytes
    // [kb, kb + 4 EW) of that group's FP8 row
    const int kg = (EW * k) / 32, kb = (4 * EW * k) % 128;
    // st: lane d = lane & 15 keeps m_ref of head HS k + d (d < HS) or E of group d - HS
    float st = (C::SLOTS <= 8 ? (lane & 7) % C::SLOTS : min(lane & 15, C::SLOTS - 1)) < HS ? -INFINITY : 0.f;
    float lsum[HS], y[NG][HS];
#pragma unroll
    for (int j = 0; j < HS; ++j) {
      lsum[j] = 0.f;
#pragma unroll
      for (int g = 0; g < NG; ++g) y[g][j] = 0.f;
    }

    // next tile's code bytes of this thread (EW bytes: 2 or 1 uint4)
    uint4 cw[EW / 16];
    bool ok_next = false;
    auto load_tile = [&](int i, int32_t raw) {
      // Codes of absent or masked tokens are never weighted (P' = 0, score discarded), so
      // they are loaded from slot 0 (padding) instead of being zeroed: no select on the load.
      const int64_t pg = page_of(i, t >> 6, raw);
      const int pos = (p0 + 2 * i) * PAGE + t;
      ok_next = pg >= 0 && pos >= lo && pos < hi;
      const int64_t slot = pg >= 0 ? pg * PAGE + (t & 63) : 0;
      const uint4* src = reinterpret_cast<const uint4*>(a.cache.codes + slot * (D / 4) + EW * k);
#pragma unroll
      for (int c = 0; c < EW / 16; ++c) cw[c] = src[c];
    };
    auto expand = [&](uint32_t(&r)[EW]) {
#pragma unroll
      for (int c = 0; c < EW / 16; ++c) {
        const uint32_t wd[4] = {cw[c].x, cw[c].y, cw[c].z, cw[c].w};
#pragma unroll
        for (int kq = 0; kq < 4; ++kq) expand_word(wd[kq], &r[16 * c + 4 * kq]);
      }
    };
    auto store_pva = [&](int buf, const uint32_t(&r)[EW]) {
      uint8_t* base = smem + C::OFF_PVA + buf * C::PVA_BUF + kg * C::PVA_GROUP;
#pragma unroll
      for (int kq = 0; kq < EW / 4; ++kq)
        *reinterpret_cast<uint4*>(base + sw128(t, kb + 16 * kq)) =
            make_uint4(r[4 * kq], r[4 * kq + 1], r[4 * kq + 2], r[4 * kq + 3]);
    };
    // prologue: tile 0 into TMEM and PV-A buffer 0, QK^T(0)
    load_tile(0, raw0);
    int32_t pg_ahead = raw1;  // page id of tile i + 2 (in the loop)
    {
      uint32_t r[EW];
      expand(r);
      tmem_st_cols<EW, C::AL_A>(tmem + lane_base + C::T_AQK + EW * k, r);
      store_pva(0, r);
      tmem_wait_st();
    }
    fence_proxy_async();
    tc_fence_before();
    mbar_arrive(&bars[B_AQK]);  // A of QK^T(0) is in TMEM
    bool ok = ok_next;
    if (ntiles > 1) load_tile(1, pg_ahead);
    pg_ahead = page_raw(2, t >> 6);

    for (int i = 0; i < ntiles; ++i) {
      const int s = i & 1;
      // -- 1. scores of tile i --
      if (alive) alive = mbar_wait(&bars[B_QK], i & 1, a.err);
      __syncwarp();
      tc_fence_after();
      if (alive) alive = mbar_wait(&bars[B_PAR + s], (i >> 1) & 1, a.err);
      float sc[NG], zz[NG];
      {
        const float* pr = reinterpret_cast<const float*>(smem + C::OFF_PAR + s * C::PAR_STAGE) + t * (NG * 2);
#pragma unroll
        for (int g2 = 0; g2 < NG / 2; ++g2) {
          const float4 pv = reinterpret_cast<const float4*>(pr)[g2];
          sc[2 * g2] = pv.x;
          zz[2 * g2] = pv.y;
          sc[2 * g2 + 1] = pv.z;
          zz[2 * g2 + 1] = pv.w;
        }
      }
#pragma unroll
      for (int g = 0; g < NG; ++g) {  // slots outside the range may hold anything
        sc[g] = ok ? sc[g] : 0.f;
        zz[g] = ok ? zz[g] : 0.f;
      }
      float s2[HS];
      {
        // A = sum_g s_g q_g.c and B = -sum_g s_g z_g sum(q_g) for heads (HS k + 2jp, +1), a
        // pair per FFMA2 (the packed FP32 pipe: two IEEE round-to-nearest FMAs per instruction)
        float2 A[HS / 2], B[HS / 2];
#pragma unroll
        for (int jp = 0; jp < HS / 2; ++jp) A[jp] = B[jp] = make_float2(0.f, 0.f);
        // -- 1b. codes of tile i+1 into TMEM (QK^T(i) has completed), in flight together with
        //        the score loads; once both have landed QK^T(i+1) may start --
        if (i + 1 < ntiles) {
#pragma unroll
          for (int c = 0; c < EW / 16; ++c) {  // 16 columns at a time (register budget)
            const uint32_t wd[4] = {cw[c].x, cw[c].y, cw[c].z, cw[c].w};
            uint32_t r[16];
#pragma unroll
            for (int kq = 0; kq < 4; ++kq) expand_word(wd[kq], &r[4 * kq]);
            tmem_st16(tmem + lane_base + C::T_AQK + EW * k + 16 * c, r);
          }
        }
        uint32_t pe[HS];
        uint32_t dq[NG][2 * HS];
#pragma unroll
        for (int g = 0; g < NG; ++g)
          tmem_ld_cols<2 * HS, C::AL_Q>(tmem + lane_base + C::T_DQK + C::GSC * g + 2 * HS * k, dq[g]);
        tmem_ld_cols<HS, C::AL_P>(tmem + lane_base + C::T_DPE + HS * k, pe);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < NG; ++g) reg_fence(dq[g]);
        reg_fence(pe);
        if (i + 1 < ntiles) {
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&bars[B_AQK]);  // A of QK^T(i+1) is in TMEM, D of QK^T(i) has been read
        }
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const float nscz = -sc[g] * zz[g];
          float2 qsv[HS / 2];  // the group sums of the query for the head pairs
          if constexpr (HS % 4 == 0) {
#pragma unroll
            for (int u = 0; u < HS / 4; ++u) {
              const float4 q4v = *reinterpret_cast<const float4*>(F + C::F_QSUM + g * H + HS * k + 4 * u);
              qsv[2 * u] = make_float2(q4v.x, q4v.y);
              qsv[2 * u + 1] = make_float2(q4v.z, q4v.w);
            }
          } else {
#pragma unroll
            for (int jp = 0; jp < HS / 2; ++jp)
              qsv[jp] = *reinterpret_cast<const float2*>(F + C::F_QSUM + g * H + HS * k + 2 * jp);
          }
#pragma unroll
          for (int jp = 0; jp < HS / 2; ++jp) {
            const float2 qs = qsv[jp];
            const uint32_t* d = dq[g];
            const float2 qc = make_float2(
                fmaf(__uint_as_float(d[HS + 2 * jp]), 0.0625f, __uint_as_float(d[2 * jp])),
                fmaf(__uint_as_float(d[HS + 2 * jp + 1]), 0.0625f, __uint_as_float(d[2 * jp + 1])));
            A[jp] = __ffma2_rn(make_float2(sc[g], sc[g]), qc, A[jp]);
            B[jp] = __ffma2_rn(make_float2(nscz, nscz), qs, B[jp]);
          }
        }
        float kinv[HS];
        if constexpr (HS % 4 == 0) {
#pragma unroll
          for (int u = 0; u < HS / 4; ++u) {
            const float4 k4 = *reinterpret_cast<const float4*>(F + C::F_KINV + HS * k + 4 * u);
            kinv[4 * u] = k4.x, kinv[4 * u + 1] = k4.y, kinv[4 * u + 2] = k4.z, kinv[4 * u + 3] = k4.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < HS; ++j) kinv[j] = F[C::F_KINV + HS * k + j];
        }
#pragma unroll
        for (int j = 0; j < HS; ++j) {
          const float Aj = (j & 1) ? A[j >> 1].y : A[j >> 1].x, Bj = (j & 1) ? B[j >> 1].y : B[j >> 1].x;
          const float kj = kinv[j];
          s2[j] = ok ? fmaf(Aj, kj, __uint_as_float(pe[j]) + Bj) * sl2 : -INFINITY;
        }
      }
      mbar_arrive(&bars[B_PFREE + s]);  // params stage s has been read (sc, zz are in registers)
      // -- 2. the warp's tile maxima (its 32 tokens) of the HS heads' scores and of the NG
      //       group scales, one redux each, into the head set's table --
      {
        float hm[HS], gx[NG];
#pragma unroll
        for (int j = 0; j < HS; ++j) hm[j] = warp_max_f32(s2[j]);
#pragma unroll
        for (int g = 0; g < NG; ++g) gx[g] = warp_max_f32(sc[g]);
        float* row = F + C::F_TAB + ((s * 4 + k) * 4 + q4) * C::SLOT_PAD;
        if constexpr (HS == 4 && NG == 4) {
          if (lane == 0) {
            reinterpret_cast<float4*>(row)[0] = make_float4(hm[0], hm[1], hm[2], hm[3]);
            reinterpret_cast<float4*>(row)[1] = make_float4(gx[0], gx[1], gx[2], gx[3]);
          }
        } else {
          float v = hm[0];  // lane d < SLOTS stores slot d (values are warp-uniform)
#pragma unroll
          for (int j = 1; j < HS; ++j) v = lane == j ? hm[j] : v;
#pragma unroll
          for (int g = 0; g < NG; ++g) v = lane == HS + g ? gx[g] : v;
          if (lane < C::SLOTS) row[lane] = v;
        }
      }
      // The four warps of head set k (one per token quarter) exchange their maxima; the head
      // sets do not wait for one another.  Each set's group-scale maxima cover all 128 tokens,
      // so every set takes the same E_g decisions.
      tc_fence_before();
      named_bar_sync(4 + k, 128);
      // -- 3. lazy-rescale decisions: lane d = lane & 15 keeps m_ref of head HS k + d (d < HS)
      //       or E of group d - HS in `st`, decides from the head set's table, and the other
      //       lanes take the results by shuffle --
      float fac = 1.f, pj[HS];
      bool resc;
      {
        const int d = C::SLOTS <= 8 ? (lane & 7) % C::SLOTS : min(lane & 15, C::SLOTS - 1);
        const float* tb = F + C::F_TAB + (s * 4 + k) * 4 * C::SLOT_PAD + d;
        const float v = fmaxf(fmaxf(tb[0], tb[C::SLOT_PAD]), fmaxf(tb[2 * C::SLOT_PAD], tb[3 * C::SLOT_PAD]));
        bool ch = false;
        if (d < HS) {  // m_ref moves when the tile max exceeds it by more than kTau
          if (v > st + kTau) {
            fac = ex2_approx(st - v);
            st = v;
            ch = true;
          }
        } else if (i == 0) {
          st = group_e(v);
        } else if (v * st >= kEMax) {  // E_g moves when the largest scale times E_g reaches kEMax
          const float en = group_e(v);
          fac = pow2_ratio(en, st);
          st = en;
          ch = true;
        }
        resc = __any_sync(0xFFFFFFFFu, ch);
        // P = 2^(s - m_ref) against the (possibly moved) reference max of each head
#pragma unroll
        for (int j = 0; j < HS; ++j) {
          const float mr = __shfl_sync(0xFFFFFFFFu, st, j);
          pj[j] = ok ? ex2_approx(s2[j] - mr) : 0.f;
        }
      }
      if (resc) {
        float alpha[HS], gf[NG];
#pragma unroll
        for (int j = 0; j < HS; ++j) alpha[j] = __shfl_sync(0xFFFFFFFFu, fac, j);
#pragma unroll
        for (int g = 0; g < NG; ++g) gf[g] = __shfl_sync(0xFFFFFFFFu, fac, HS + g);
#pragma unroll
        for (int j = 0; j < HS; ++j) {
          lsum[j] *= alpha[j];
#pragma unroll
          for (int g = 0; g < NG; ++g) y[g][j] *= alpha[j] * gf[g];
        }
        if (i > 0) {  // O holds PV(0..i-1): scale the columns of this head set (warp-uniform branch)
          if (alive) alive = mbar_wait(&bars[B_PV], (i - 1) & 1, a.err);
          __syncwarp();
          tc_fence_after();
#pragma unroll
          for (int g = 0; g < NG; ++g) {
            uint32_t v[2 * HS];
            const uint32_t ta = tmem + lane_base + C::T_O + C::GSC * g + 2 * HS * k;
            tmem_ld_cols<2 * HS, C::AL_Q>(ta, v);
            tmem_wait_ld();
            reg_fence(v);
#pragma unroll
            for (int c = 0; c < 2 * HS; ++c) v[c] = __float_as_uint(__uint_as_float(v[c]) * (alpha[c % HS] * gf[g]));
            tmem_st_cols<2 * HS, C::AL_Q>(ta, v);
          }
          tmem_wait_st();
          tc_fence_before();
        }
      }
#pragma unroll
      for (int j = 0; j < HS; ++j) lsum[j] += pj[j];
      // -- 3b. P' = P s_g E_g as hi + lo / 16 (two E4M3 terms; the residual is scaled by 16 to
      //        stay in E4M3's normal range); y sums exactly the value the tensor core sees --
      uint8_t* pb = smem + C::OFF_PB + s * C::PB_BUF;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const float se = sc[g] * __shfl_sync(0xFFFFFFFFu, st, HS + g);
        uint32_t pw[HS / 2];  // bytes [hi of the HS heads, lo of the HS heads]
#pragma unroll
        for (int w = 0; w < HS / 2; ++w) pw[w] = 0;
#pragma unroll
        for (int jp = 0; jp < HS / 2; ++jp) {
          const __half2 hx = __floats2half2_rn(pj[2 * jp] * se, pj[2 * jp + 1] * se);
          const uint32_t hq = half2_to_e4m3x2(hx);
          const __half2 hf = e4m3x2_to_half2(hq);
          const uint32_t lq = half2_to_e4m3x2(__hmul2(__hsub2(hx, hf), __float2half2_rn(16.f)));
          const float2 v = __half22float2(__hfma2(e4m3x2_to_half2(lq), __float2half2_rn(0.0625f), hf));
          y[g][2 * jp] = fmaf(v.x, zz[g], y[g][2 * jp]);
          y[g][2 * jp + 1] = fmaf(v.y, zz[g], y[g][2 * jp + 1]);
          pw[(2 * jp) / 4] |= hq << (8 * ((2 * jp) % 4));
          pw[(HS + 2 * jp) / 4] |= lq << (8 * ((HS + 2 * jp) % 4));
        }
        uint8_t* prow = pb + g * C::PB_GROUP;
        if constexpr (C::PB_ROW == 32) {
          if constexpr (HS / 2 == 2) {
            *reinterpret_cast<uint2*>(prow + sw32(t, 2 * HS * k)) = make_uint2(pw[0], pw[1]);
          } else {
#pragma unroll
            for (int w = 0; w < HS / 2; ++w) *reinterpret_cast<uint32_t*>(prow + sw32(t, 2 * HS * k + 4 * w)) = pw[w];
          }
        } else {
#pragma unroll
          for (int w = 0; w < HS / 2; ++w) *reinterpret_cast<uint32_t*>(prow + sw128(t, 2 * HS * k + 4 * w)) = pw[w];
        }
      }
      // -- 4. the PV-A tile of i+1 into buffer (i+1) & 1, last read by PV(i-1).  PV(i-1) is
      //       waited for on every tile (the last one too): PREADY(i) then cannot complete
      //       before the MMA warp has taken PREADY(i-1), so its parity wait never aliases. --
      __syncwarp();  // the tcgen05.ld below is warp-collective
      if (i + 1 < ntiles) {
        uint32_t r[EW];  // the FP8 codes of tile i+1, as 1b wrote them to TMEM (read before the wait)
        tmem_ld_cols<EW, C::AL_A>(tmem + lane_base + C::T_AQK + EW * k, r);
        tmem_wait_ld();
        reg_fence(r);
        if (alive && i >= 1) alive = mbar_wait(&bars[B_PV], (i - 1) & 1, a.err);
        tc_fence_after();
        store_pva((i + 1) & 1, r);
        ok = ok_next;
        if (i + 2 < ntiles) {
          load_tile(i + 2, pg_ahead);
          pg_ahead = page_raw(i + 3, t >> 6);
        }
      } else if (alive && i >= 1) {
        alive = mbar_wait(&bars[B_PV], (i - 1) & 1, a.err);
      }
      fence_proxy_async();  // the P' and PV-A stores above, for the tensor core's reads
      mbar_arrive(&bars[B_PREADY]);  // P'(i), the PV-A tile of i+1 and a rescaled O are ready;
                                     // params stage i & 1 has been read
    }
    // -- final: sum P and sum P' z over the warp's 32 tokens --
    if constexpr (HS == 4 && NG == 4) {
      // Transposed butterfly: at the xor-16, 8, 4, 2 steps each lane keeps half of its
      // remaining values and adds its partner's copy of them (the same pairing per value as
      // five plain xor steps), so a value ends in the lanes whose bits 4..1 spell its index.
      float v[16];  // y[g][j] at index 4g + j
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) v[4 * g + j] = y[g][j];
#pragma unroll
      for (int half = 8, o = 16; half >= 1; half >>= 1, o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float keep = up ? v[i + half] : v[i], send = up ? v[i] : v[i + half];
          v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
        }
      }
      v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], 1);
      const int idx = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
      if ((lane & 1) == 0) F[C::F_FINY + ((idx >> 2) * H + 4 * k + (idx & 3)) * 4 + q4] = v[0];
      float l[4] = {lsum[0], lsum[1], lsum[2], lsum[3]};
#pragma unroll
      for (int half = 2, o = 16; half >= 1; half >>= 1, o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float keep = up ? l[i + half] : l[i], send = up ? l[i] : l[i + half];
          l[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
        }
      }
#pragma unroll
      for (int o = 4; o >= 1; o >>= 1) l[0] += __shfl_xor_sync(0xFFFFFFFFu, l[0], o);
      if ((lane & 7) == 0) F[C::F_FINL + (4 * k + ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1)) * 4 + q4] = l[0];
    } else {
      // plain xor reductions (the same pairing per value as the butterfly above)
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int j = 0; j < HS; ++j) {
          const float r = warp_sum(y[g][j]);
          if (lane == 0) F[C::F_FINY + (g * H + HS * k + j) * 4 + q4] = r;
        }
#pragma unroll
      for (int j = 0; j < HS; ++j) {
        const float r = warp_sum(lsum[j]);
        if (lane == 0) F[C::F_FINL + (HS * k + j) * 4 + q4] = r;
      }
    }
    named_bar_sync(3, TOK_THREADS);
    float lt[HS];  // sum P over the split per head HS k + j
#pragma unroll
    for (int j = 0; j < HS; ++j) {
      const float4 q = *reinterpret_cast<const float4*>(F + C::F_FINL + (HS * k + j) * 4);
      lt[j] = ((0.f + q.x) + q.y + q.z) + q.w;  // quarter order 0..3, as the scalar sum
    }
    float E[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) E[g] = __shfl_sync(0xFFFFFFFFu, st, HS + g);
    {
      float m_ref[HS];
#pragma unroll
      for (int j = 0; j < HS; ++j) m_ref[j] = __shfl_sync(0xFFFFFFFFu, st, j);
      if (q4 == 0 && lane == 0) {
#pragma unroll
        for (int j = 0; j < HS; ++j)
          a.part_lse[(static_cast<int64_t>(b) * H + HS * k + j) * S + split] =
              lt[j] > 0.f ? (m_ref[j] + __log2f(lt[j])) * kLn2 : -INFINITY;
      }
    }
    // -- O rows of this lane quarter (M row = permuted element), columns of head set k --
    if (alive) alive = mbar_wait(&bars[B_PV], (ntiles - 1) & 1, a.err);
    __syncwarp();
    tc_fence_after();
    const float rs = ((t >> 2) & 1) ? 128.f : 512.f;  // 2^9 / (1 or 4): the element's code weight
    float il[HS], ie[NG];  // 1 / sum P per head (0 for an empty split), 1 / E_g (exact: powers of two)
#pragma unroll
    for (int j = 0; j < HS; ++j) il[j] = lt[j] > 0.f ? __frcp_rn(lt[j]) : 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) ie[g] = __int_as_float((254 << 23) - __float_as_int(E[g]));  // 2^-e for E = 2^e
    float* po = a.part_o + (static_cast<int64_t>(b) * H * S + split) * D + kperm(t);
    const int hs = S * D;  // head stride of part_o
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      uint32_t v[2 * HS];
      tmem_ld_cols<2 * HS, C::AL_Q>(tmem + lane_base + C::T_O + C::GSC * g + 2 * HS * k, v);
      tmem_wait_ld();
      reg_fence(v);
#pragma unroll
      for (int j = 0; j < HS; ++j) {
        const float4 q = *reinterpret_cast<const float4*>(F + C::F_FINY + (g * H + HS * k + j) * 4);
        const float yy = ((0.f + q.x) + q.y + q.z) + q.w;
        const float dh = fmaf(__uint_as_float(v[HS + j]), 0.0625f, __uint_as_float(v[j]));
        po[(HS * k + j) * hs + 128 * g] = (dh * rs - yy) * (il[j] * ie[g]);
      }
    }
    tc_fence_before();
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      // ---- MMA issue: QK^T(i) once its codes are in TMEM, PV(i-1) once P'(i-1) is ready -------
      const uint64_t dq0 = sw128_kmajor_desc(smem_u32(smem + C::OFF_QB));
      const uint64_t dk0 = DR == 64 ? sw128_kmajor_desc(smem_u32(smem + C::OFF_KPE))
                                    : sw64_kmajor_desc(smem_u32(smem + C::OFF_KPE));
      const uint64_t dqp = DR == 64 ? sw128_kmajor_desc(smem_u32(smem + C::OFF_QPE))
                                    : sw64_kmajor_desc(smem_u32(smem + C::OFF_QPE));
      const uint64_t dpa0 = mn_major_desc(smem_u32(smem + C::OFF_PVA), 128);
      const uint64_t dpb0 = mn_major_desc(smem_u32(smem + C::OFF_PB), C::PB_ROW);
      for (int i = 0; i < ntiles; ++i) {
        if (alive) alive = mbar_wait(&bars[B_AQK], i & 1, a.err);
        if (alive) alive = mbar_wait(&bars[B_KPE + (i & 1)], (i >> 1) & 1, a.err);
        tc_fence_after();
        issue_qk(i, dq0, dk0, dqp);
        if (i >= 1) {
          if (alive) alive = mbar_wait(&bars[B_PREADY], (i - 1) & 1, a.err);
          tc_fence_after();
          issue_pv(i - 1, dpa0, dpb0);
        }
      }
      if (alive) alive = mbar_wait(&bars[B_PREADY], (ntiles - 1) & 1, a.err);
      tc_fence_after();
      issue_pv(ntiles - 1, dpa0, dpb0);
    }
  } else if (lane == 0) {
    // ---- producer: k_pe TMA and params bulk copies into their 2-stage rings, L2 prefetch -----
    prefetch_tensormap(&tm_rope);
    // page ids of tiles i+1 .. i+5, fetched five tiles ahead
    int32_t r1a = page_raw(1, 0), r1b = page_raw(1, 1), r2a = page_raw(2, 0), r2b = page_raw(2, 1);
    int32_t r3a = page_raw(3, 0), r3b = page_raw(3, 1), r4a = page_raw(4, 0), r4b = page_raw(4, 1);
    int32_t r5a = page_raw(5, 0), r5b = page_raw(5, 1);
    {
      const int32_t r0a = page_raw(0, 0), r0b = page_raw(0, 1);
      issue_kpe(0, r0a, r0b);
      issue_params(0, r0a, r0b);
    }
    if (ntiles > 1) {
      issue_kpe(1, r1a, r1b);
      issue_params(1, r1a, r1b);
    }
    if (ntiles > 2) prefetch_tile(2, r2a, r2b);
    if (ntiles > 3) prefetch_tile(3, r3a, r3b);
    for (int i = 0; i < ntiles; ++i) {
      if (i + 1 < ntiles && i >= 1) {  // params stage (i+1) & 1 held tile i-1
        if (alive) alive = mbar_wait(&bars[B_PFREE + ((i - 1) & 1)], ((i - 1) >> 1) & 1, a.err);
        issue_params(i + 1, r1a, r1b);
      }
      if (i + 2 < ntiles) {  // k_pe stage i & 1 is free once QK^T(i) has completed
        if (alive) alive = mbar_wait(&bars[B_KFREE + (i & 1)], (i >> 1) & 1, a.err);
        issue_kpe(i + 2, r2a, r2b);
      }
      if (i + 4 < ntiles) prefetch_tile(i + 4, r4a, r4b);
      r1a = r2a, r1b = r2b, r2a = r3a, r2b = r3b, r3a = r4a, r3b = r4b, r4a = r5a, r4b = r5b;
      r5a = page_raw(i + 6, 0);
      r5b = page_raw(i + 6, 1);
    }
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  // Launched as a programmatic dependent of the window kernel: finish only after that grid
  // has, so that the merge kernel (waiting on this grid) sees the window partials.  Without
  // a programmatic launch this returns at once.
  grid_dependency_wait();
}

}  // namespace tc

static int map_rope(CUtensorMap* map, const void* base, uint64_t rows, int dr) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ROLAQ_ECUDA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(dr), rows};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(dr * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(dr), static_cast<cuuint32_t>(tc::PAGE)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = dr == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ROLAQ_OK : ROLAQ_ECUDA;
}

bool decode_tc_supported(const DecodeArgs& a, int heads) {
  const int d = a.cache.latent_dim, dr = a.cache.rope_dim;
  const bool shape = (d == 512 && dr == 64 && (heads == 16 || heads == 8)) ||
                     (d == 256 && dr == 32 && (heads == 40 || heads == 16));
  return shape && (a.q_sh % 8) == 0 && (a.q_sb % 8) == 0 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0;
}

template <int D, int DR, int H>
static int launch_tc_t(const DecodeArgs& a, cudaStream_t s, bool dependent) {
  using C = tc::Cfg<D, DR, H>;
  CUtensorMap mr;
  int rc = map_rope(&mr, a.cache.rope, static_cast<uint64_t>(a.cache.num_slots), DR);
  if (rc != ROLAQ_OK) return rc;
  static const bool attr_ok = cudaFuncSetAttribute(tc::decode_tc_kernel<D, DR, H>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)C::SMEM) == cudaSuccess;
  if (!attr_ok) return ROLAQ_ECUDA;
  dim3 grid(a.num_splits, a.batch);
  if (!dependent) {
    tc::decode_tc_kernel<D, DR, H><<<grid, tc::THREADS, C::SMEM, s>>>(mr, a);
    return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
  }
  // a programmatic dependent of the kernel before it in the stream (the window split)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(tc::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, tc::decode_tc_kernel<D, DR, H>, mr, a) != cudaSuccess) return ROLAQ_ECUDA;
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

int launch_decode_tc(const DecodeArgs& a, int heads, cudaStream_t s, bool dependent) {
  const int d = a.cache.latent_dim;
  if (d == 512)
    return heads == 16 ? launch_tc_t<512, 64, 16>(a, s, dependent) : launch_tc_t<512, 64, 8>(a, s, dependent);
  return heads == 40 ? launch_tc_t<256, 32, 40>(a, s, dependent) : launch_tc_t<256, 32, 16>(a, s, dependent);
}

}  // namespace rolaq
