// Per-head projections on either side of the absorbed MLA decode, on tcgen05 (sm_100a):
//   absorbed query     q[b, h, n]     = sum_k q_nope[b, h, k] w_kc[h][n][k]   (n < D), and the
//                      rope tail      q[b, h, D + r] = q_pe[b, h, r]            (the concat)
//   output projection  out[b, h, v]   = sum_e o[b, h, e] w_vc[h][v][e]
// BF16 inputs, FP32 accumulation in TMEM, BF16 outputs.
//
// Reference: deployment/patches/rolaq_sglang.patch:205-248, 261-274 -- the DeepSeek MLA
// forward's torch.bmm(q_nope, w_kc) + cat([q_nope_out, q_pe]) before the packed decode and
// torch.bmm(attn_output, w_vc) after it, with the read rotation folded into w_kc / w_vc by
// fold_read_rotation (deployment/sglang/srt/mem_cache/rolaq_mla.py:56-71), so that the
// decode's queries and outputs stay in the rotated latent frame.  The weights are taken in
// the layout SGLang keeps them in for its bmm (w_kc stored [H, D, Dn], w_vc [H, Dv, D]:
// the reduced dimension contiguous), which is the K-major B operand of the MMA.
//
// One CTA per (output tile of up to 256 columns, head, 128 batch rows): warp 0 streams
// 64-wide K chunks of the activation rows (TMA on a 3-D map over (K, head, batch row); rows
// past the batch read as zero) and of the head's weight rows (TMA, 2-D) through a 3-stage
// ring; one thread of warp 1 issues kind::f16 MMAs (M = 128 batch rows, N = the tile) into a
// TMEM accumulator; warps 2..5 (one per TMEM lane quarter) read it back, round to BF16 and
// store their rows.
#include "kernels.cuh"

namespace rolaq {
namespace proj {

constexpr int TM = 128, TK = 64, STAGES = 3;
constexpr int THREADS = 6 * 32;
constexpr int A_CHUNK = TM * TK * 2;  // 16 KB

template <int NT>
struct PCfg {
  static constexpr int B_CHUNK = NT * TK * 2;
  static constexpr int STAGE = A_CHUNK + B_CHUNK;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE + 1024 + 128;
  static_assert(NT == 64 || NT == 128 || NT == 256, "N tile");
};

template <int NT>
__global__ void __launch_bounds__(THREADS, 1)
    proj_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, const ProjArgs a) {
  using C = PCfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * NT, h = blockIdx.y, b0 = blockIdx.z * TM;
  const int nk = a.k / TK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
    prefetch_tensormap(&tm_x);
    prefetch_tensormap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, NT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer ----
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % STAGES;
        if (kc >= STAGES && !mbar_wait(&empty[s], ((kc / STAGES) - 1) & 1, a.err)) break;
        uint8_t* st = smem + s * C::STAGE;
        mbar_expect_tx(&full[s], C::STAGE);
        tma_load_3d(st, &tm_x, &full[s], kc * TK, h, b0);
        tma_load_2d(st + A_CHUNK, &tm_w, &full[s], kc * TK, h * a.n + n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issue ----
      const uint32_t idesc = idesc_bf16(TM, NT);
      const uint64_t d0 = sw128_kmajor_desc(smem_u32(smem));
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % STAGES;
        if (!mbar_wait(&full[s], (kc / STAGES) & 1, a.err)) break;
        tc_fence_after();
        const uint64_t da = d0 + static_cast<uint64_t>((s * C::STAGE) >> 4);
        const uint64_t db = da + static_cast<uint64_t>(A_CHUNK >> 4);
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) umma_bf16_ss(tmem, da + 2 * kk, db + 2 * kk, idesc, (kc | kk) != 0);
        umma_commit(&empty[s]);
      }
      // Also when a wait gave up: the epilogue then finds the phase complete, and the
      // timeout bit in the caller's err word marks the output as invalid.
      umma_commit(tfull);
    }
  } else {  // ---- epilogue: warps 2..5, TMEM lane quarter warp & 3 ----
    const int quad = warp & 3;
    const int b = b0 + 32 * quad + lane;
    const bool live = mbar_wait(tfull, 0, a.err);
    tc_fence_after();
    uint16_t* orow = a.out + static_cast<int64_t>(b) * a.o_sb + static_cast<int64_t>(h) * a.o_sh + n0;
#pragma unroll 1
    for (int c = 0; c < NT; c += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * quad) << 16) + c, r);
      tmem_wait_ld();
      reg_fence(r);
      if (live && b < a.batch) {
        uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[j] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * j]), __uint_as_float(r[8 * j + 1])),
                              pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3])),
                              pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5])),
                              pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7])));
      }
    }
    if (a.pe != nullptr && blockIdx.x == 0 && b < a.batch) {  // the rope tail of the query row
      const uint4* src = reinterpret_cast<const uint4*>(a.pe + static_cast<int64_t>(b) * a.pe_sb +
                                                        static_cast<int64_t>(h) * a.pe_sh);
      uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(b) * a.o_sb +
                                            static_cast<int64_t>(h) * a.o_sh + a.n);
      for (int j = 0; j < a.dr / 8; ++j) dst[j] = src[j];
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, NT);
  }
}

}  // namespace proj

int launch_proj(const ProjArgs& a, cudaStream_t s) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ROLAQ_ECUDA;
  CUtensorMap mx, mw;
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(a.k), static_cast<cuuint64_t>(a.heads),
                          static_cast<cuuint64_t>(a.batch)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(a.x_sh) * 2, static_cast<cuuint64_t>(a.x_sb) * 2};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(proj::TK), 1, static_cast<cuuint32_t>(proj::TM)};
    cuuint32_t estr[3] = {1, 1, 1};
    if (fn(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(a.x), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return ROLAQ_ECUDA;
  }
  const int nt = a.n >= 256 ? 256 : a.n;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k), static_cast<cuuint64_t>(a.heads) * a.n};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(proj::TK), static_cast<cuuint32_t>(nt)};
    cuuint32_t estr[2] = {1, 1};
    if (fn(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a.w), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return ROLAQ_ECUDA;
  }
  const dim3 grid(static_cast<unsigned>(a.n / nt), static_cast<unsigned>(a.heads),
                  static_cast<unsigned>((a.batch + proj::TM - 1) / proj::TM));
  // Attributes set once per process (graph capture records launches, not API calls).
  static const bool attr256 = cudaFuncSetAttribute(proj::proj_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)proj::PCfg<256>::SMEM) == cudaSuccess;
  static const bool attr128 = cudaFuncSetAttribute(proj::proj_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)proj::PCfg<128>::SMEM) == cudaSuccess;
  static const bool attr64 = cudaFuncSetAttribute(proj::proj_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)proj::PCfg<64>::SMEM) == cudaSuccess;
  if (nt == 256) {
    if (!attr256) return ROLAQ_ECUDA;
    proj::proj_kernel<256><<<grid, proj::THREADS, proj::PCfg<256>::SMEM, s>>>(mx, mw, a);
  } else if (nt == 128) {
    if (!attr128) return ROLAQ_ECUDA;
    proj::proj_kernel<128><<<grid, proj::THREADS, proj::PCfg<128>::SMEM, s>>>(mx, mw, a);
  } else {
    if (!attr64) return ROLAQ_ECUDA;
    proj::proj_kernel<64><<<grid, proj::THREADS, proj::PCfg<64>::SMEM, s>>>(mx, mw, a);
  }
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

}  // namespace rolaq
