/*
 * rolaq_b200.h -- C ABI of the B200 (sm_100a) packed-INT2 MLA content-cache path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t, returns
 * an int status (ROLAQ_OK or a negative ROLAQ_E* code, with a message available from
 * rolaq_last_error()), never allocates device memory, never synchronises the stream
 * and never throws.  All buffers are owned by the caller.  Calls on different
 * streams are independent; calls that write the same cache buffers must be ordered
 * by the caller.  Problems that can only be seen on the device (a slot or page index
 * out of range, a wait that ran out of time) are OR-ed into the caller's optional
 * `err` word (ROLAQ_DEV_* bits) instead of faulting.
 *
 * Cache layout of one layer (the "pool"), shared by the writer and the reader:
 *   codes  uint8 [num_slots, D/4]      code of latent element j at byte j/4, bits 2*(j%4)
 *   params f32   [num_slots, D/128, 2] (scale, zero) per 128-element group
 *   rope   bf16  [num_slots, Dr]       k_pe, unquantized
 *   hp     bf16  [num_ring_rows, D]    rotated latents of the s4r16 window tokens
 *   rows   i32   [num_slots]           ring row of a slot, or -1   (shared by layers)
 *   owners i32   [num_ring_rows]       slot that owns a ring row  (shared by layers)
 * with num_ring_rows = 1 + max_reqs * (sink + recent).  Slot 0 backs CUDA-graph
 * padding.  Reader pages are 64 consecutive slots.
 *
 * The reference interfaces each entry point replaces are cited per function
 * (paths inside noforit/mla_kv_quant).
 */
#ifndef ROLAQ_B200_H_
#define ROLAQ_B200_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ROLAQ_OK 0
#define ROLAQ_EINVAL (-1)       /* bad pointer, size, stride or alignment */
#define ROLAQ_EUNSUPPORTED (-2) /* shape outside what the kernels implement */
#define ROLAQ_ECUDA (-3)        /* a CUDA runtime call or kernel launch failed */

/* Bits OR-ed into the optional device-side `err` word. */
#define ROLAQ_DEV_BAD_SLOT 1    /* a slot index outside [0, num_slots) was skipped */
#define ROLAQ_DEV_BAD_PAGE 2    /* a page index outside the pool was skipped */
#define ROLAQ_DEV_TIMEOUT 4     /* a bounded wait on an mbarrier gave up */
#define ROLAQ_DEV_BAD_REQ 8     /* seq_len larger than the page table allows */
#define ROLAQ_DEV_PEER_TIMEOUT 16 /* a bounded wait for another rank's partial gave up */

/* One layer of the packed cache plus the shared slot/ring maps. */
typedef struct rolaq_layer_cache {
  uint8_t* codes;
  float* params;
  uint16_t* rope;
  uint16_t* hp;      /* may be NULL when sink + recent == 0 */
  int32_t* rows;     /* may be NULL when sink + recent == 0 */
  int32_t* owners;   /* may be NULL when sink + recent == 0 */
  int64_t num_slots;
  int64_t num_ring_rows;
  int32_t latent_dim; /* D: 256 or 512 */
  int32_t rope_dim;   /* Dr: 32 or 64 */
  int32_t sink;       /* P */
  int32_t recent;     /* W */
  int64_t max_reqs;
} rolaq_layer_cache;

/* Codec families of the INT2 writer. */
#define ROLAQ_CODEC_LLOYD 0   /* learned Lloyd grid (mla_quant/oscar.py:120-144) */
#define ROLAQ_CODEC_UNIFORM 1 /* OSCAR's uniform min/max baseline (mla_quant/oscar.py:91-101) */

/* Scalars of the INT2 codec, already rounded to FP32 the way the calling path rounds
 * them (mla_quant/quantizer.py:31-35 for the HF path,
 * deployment/sglang/QuantKernel/mla_fused_writer.py:158-164 for serving).
 * family ROLAQ_CODEC_UNIFORM ignores the three scalars: per 128-group
 * scale = (max - min) / 3 (1 when |max - min| <= 1e-8), code = clamp(round_half_even(
 * (x - min) / scale), 0, 3), and the stored zero is FP32(-min / scale). */
typedef struct rolaq_codec {
  float threshold;    /* t:  code = [n >= -t] + [n >= 0] + [n >= t] */
  float scale_factor; /* FP32((span / 3) * gain); scale = scale_factor * std */
  float zero_const;   /* FP32(-C0 / (span / 3)); zero = zero_const - mean / scale */
  int32_t family;     /* ROLAQ_CODEC_LLOYD or ROLAQ_CODEC_UNIFORM */
} rolaq_codec;

/* Library version (major * 10000 + minor * 100 + patch). */
int rolaq_version(void);

/* Message for the last non-OK status returned on this host thread. */
const char* rolaq_last_error(void);

/* ROLAQ_OK when the current device is an sm_100 part this library was built for. */
int rolaq_check_device(void);

/*
 * Codec + scatter of already-rotated FP32 rows: codes[slot] and params[slot] for
 * every row i with 0 <= slots[i] < num_slots.
 * Replaces scatter_pack_rows(x, slots, codes_buf, params_buf, group_size, lloyd_max,
 * bits=2, quantizer_params) (deployment/patches/rolaq_sglang.patch:9-34; body in the
 * un-vendored upstream mla_latent_int2.py).
 *   x      f32 [n, D] with row stride ldx (elements)
 *   slots  int32 or int64 [n] (slots_are_int64 selects)
 */
int rolaq_scatter_pack_rows(const float* x, int64_t ldx, const void* slots, int slots_are_int64,
                            int64_t n, int32_t latent_dim, int32_t group_size, rolaq_codec codec,
                            uint8_t* codes, float* params, int64_t num_slots, int32_t* err,
                            cudaStream_t stream);

/*
 * Auxiliary stores of the decode writer: rope[slot] = k_pe; for protected rows
 * (pos < sink or pos >= seq_len - recent, 0 <= req < max_reqs, slot > 0) the BF16
 * rotated latent goes to ring row r = 1 + req*(sink+recent) + (pos < sink ? pos :
 * sink + (pos - sink) % recent), owners[r] = slot, rows[slot] = r; other rows with
 * slot > 0 get rows[slot] = -1.  positions == NULL means pos = seq_len - 1.
 * Replaces _aux (deployment/sglang/QuantKernel/mla_fused_writer.py:16-51).
 *   c      f32 [n, D] rotated rows, row stride ldc
 *   k_pe   bf16 [n, Dr], row stride ld_pe
 *   seq_lens / req_idx / positions: int32 or int64 [n] (the *_is64 flags select)
 */
int rolaq_write_aux(const float* c, int64_t ldc, const uint16_t* k_pe, int64_t ld_pe,
                    const int64_t* slots, const void* seq_lens, int seq_lens_is64,
                    const void* req_idx, int req_idx_is64, const void* positions,
                    int positions_is64, int64_t n, const rolaq_layer_cache* cache, int32_t* err,
                    cudaStream_t stream);

/*
 * Fused writer: c = c_kv @ R on tcgen05 tensor cores (BF16 x BF16 -> FP32 in
 * TMEM, operands staged by TMA), then the codec, the packed scatter, the BF16 k_pe
 * store and the ring stores of rolaq_write_aux, in one launch.  Decode (one row per
 * request, positions == NULL) and prefill (explicit positions) both go through it.
 * Replaces try_fast_decode_store(pool, layer_id, loc, c_kv, k_pe) / _pack_and_aux
 * (deployment/sglang/QuantKernel/mla_fused_writer.py:54-224), which ran an FP32
 * cuBLAS GEMM and then a Triton kernel.
 *   c_kv    bf16 [n, D], row stride ld_ckv (elements, multiple of 8, 16-byte aligned)
 *   rot_t   bf16 [D, D] row-major transpose of the effective rotation:
 *           rot_t[o][k] = bf16(R[k][o]) (rolaq_mla.py:69 rounds R to BF16)
 *   seq_lens / req_idx may be NULL (no ring stores); see rolaq_write_aux.
 *   k_pe may be NULL (no rope stores; cache->rope may then be NULL too).
 */
int rolaq_fused_write(const uint16_t* c_kv, int64_t ld_ckv, const uint16_t* k_pe, int64_t ld_pe,
                      const int64_t* slots, const void* seq_lens, int seq_lens_is64,
                      const void* req_idx, int req_idx_is64, const void* positions,
                      int positions_is64, int64_t n, const uint16_t* rot_t, rolaq_codec codec,
                      const rolaq_layer_cache* cache, int32_t* err, cudaStream_t stream);

/*
 * Plain rotation GEMM on tcgen05: out[i][o] = sum_k x[i][k] * w[o][k], BF16 inputs,
 * FP32 accumulation, FP32 and/or BF16 output (either pointer may be NULL).  Used
 * for the un-rotation of the HF quantize-dequantize path
 * (mla_quant/quantizer.py:117-121: `dequantized.float() @ effective.T`).
 *   x  bf16 [n, D] (row stride ldx), w bf16 [D, D] row-major, out row stride ld_out.
 */
int rolaq_rotate_rows(const uint16_t* x, int64_t ldx, int64_t n, int32_t latent_dim,
                      const uint16_t* w, float* out_f32, uint16_t* out_bf16, int64_t ld_out,
                      cudaStream_t stream);

/*
 * Dequantize packed rows: out[i] = (code - zero) * scale of slot slots[i] (or of row
 * i when slots == NULL), FP32 and/or BF16 (mla_quant/oscar.py:144).
 */
int rolaq_dequant_rows(const uint8_t* codes, const float* params, const void* slots,
                       int slots_are_int64, int64_t n, int32_t latent_dim, int64_t num_slots,
                       float* out_f32, uint16_t* out_bf16, int64_t ld_out, int32_t* err,
                       cudaStream_t stream);

/*
 * quant[i] = max(splits[i] - 1, 1); merge[i] = quant[i] + 1.
 * Replaces prepare_gf_splits (deployment/patches/rolaq_sglang.patch:81-92).
 */
int rolaq_prepare_gf_splits(const int32_t* splits, int32_t* quant, int32_t* merge, int64_t n,
                            cudaStream_t stream);

/*
 * Absorbed MLA decode attention over the packed INT2 cache.
 * Token t of request b lives in slot page_table[b][t / 64] * 64 + t % 64.  Window
 * tokens (t < sink or t >= seq_len - recent) are read from their BF16 ring row when
 * owners[rows[slot]] == slot, else from the INT2 codes; all other tokens from the
 * INT2 codes.  The INT2 range is cut into num_splits page-aligned splits plus one
 * window split; each writes its (lse, o) partial; the partials are LSE-merged into
 * out (BF16, rotated latent frame) and out_lse (natural log, may be NULL).
 * Replaces packed_mla_decode_gf_fwd + _fwd_hp_window_stage1 + stage 2 (upstream,
 * called at deployment/patches/rolaq_sglang.patch:51-111).
 *   q          bf16 [B, H, D + Dr] with strides (q_stride_b, q_stride_h) in elements;
 *              q[..., :D] is q_nope_out in the rotated frame, q[..., D:] is q_pe
 *   page_table int32 [B, max_pages] (row stride pt_stride)
 *   seq_lens   int32 [B]
 *   token_range int32 [B, 2] or NULL: attend only to positions in [start, end) of each
 *              request (sequence-split decode: each rank owns one contiguous slice;
 *              window tokens count only where they fall inside the slice)
 *   part_o     f32 [B, H, num_splits + 1, D]  scratch (the reference's attn_logits)
 *   part_lse   f32 [B, H, num_splits + 1]     scratch (the reference's attn_lse)
 *   out        bf16 [B, H, D] with strides (out_stride_b, out_stride_h)
 *              (NULL: only the split partials are written, the window split's at index
 *              num_splits, for a caller that merges them itself, e.g. across ranks)
 * Supported: H = 16 with D = 512, Dr = 64; H = 40 with D = 256, Dr = 32 (any H that
 * is a multiple of 8 up to 64 with D in {256, 512}).
 */
int rolaq_packed_decode(const uint16_t* q, int64_t q_stride_b, int64_t q_stride_h, int32_t batch,
                        int32_t heads, const rolaq_layer_cache* cache, const int32_t* page_table,
                        int64_t pt_stride, int32_t max_pages, const int32_t* seq_lens,
                        const int32_t* token_range, float sm_scale, int32_t num_splits,
                        float* part_o, float* part_lse,
                        uint16_t* out, int64_t out_stride_b, int64_t out_stride_h, float* out_lse,
                        int32_t* err, cudaStream_t stream);

/*
 * rolaq_packed_decode with the split partials (part_o, part_lse) in a fixed 32 MiB
 * device array of this library instead of caller scratch: for callers that cannot
 * allocate at decode time.  No counterpart in the reference (its decode always takes
 * attn_logits / attn_lse from the caller).  Limit: batch * heads * (num_splits + 1) *
 * (latent_dim + 1) <= rolaq_packed_decode_static_capacity() floats, else ROLAQ_EINVAL.
 * The first call on a device resolves the array's address (cudaGetSymbolAddress) and
 * should come before any stream capture; nothing in the array needs to start at zero;
 * calls that overlap in time on one device share the array and race.
 */
int64_t rolaq_packed_decode_static_capacity(void);
int rolaq_packed_decode_static(const uint16_t* q, int64_t q_stride_b, int64_t q_stride_h, int32_t batch,
                               int32_t heads, const rolaq_layer_cache* cache, const int32_t* page_table,
                               int64_t pt_stride, int32_t max_pages, const int32_t* seq_lens,
                               const int32_t* token_range, float sm_scale, int32_t num_splits,
                               uint16_t* out, int64_t out_stride_b, int64_t out_stride_h, float* out_lse,
                               int32_t* err, cudaStream_t stream);

/*
 * The reader's page table from SGLang's token -> slot map, in one launch (capture-safe):
 * page_table[b][p] = req_to_token[req_pool_indices[b]][64 p] / 64 for p < ceil(seq_lens[b] / 64)
 * when those tokens sit in 64 consecutive slots starting at a multiple of 64, else -1 with
 * ROLAQ_DEV_BAD_PAGE in *err; pages past the request are -1.  seq_lens_out (int32 [B], may be
 * NULL) receives the lengths as the reader takes them.  Replaces the request -> token
 * indexing that TritonAttnBackend.forward_decode hands to packed_mla_decode_gf_fwd
 * (deployment/patches/rolaq_sglang.patch:51-72; forward_batch.req_to_token_pool.req_to_token,
 * req_pool_indices, seq_lens).
 *   req_to_token      int32 [max_reqs, rt_stride], rt_stride >= 64 * max_pages
 *   req_pool_indices  int32 or int64 [B];  seq_lens int32 or int64 [B]
 *   page_table        int32 [B, pt_stride], pt_stride >= max_pages
 */
int rolaq_page_table_from_req_to_token(const int32_t* req_to_token, int64_t rt_stride, const void* req_pool_indices,
                                       int req_is64, const void* seq_lens, int seq_lens_is64, int64_t batch,
                                       int32_t max_pages, int32_t* page_table, int64_t pt_stride,
                                       int32_t* seq_lens_out, int32_t* err, cudaStream_t stream);

/*
 * Absorbed query of the MLA decode, on tcgen05: per request b and head h,
 *   q_out[b][h][n]              = sum_k q_nope[b][h][k] * w_kc[h][n][k]   (n < latent_dim)
 *   q_out[b][h][latent_dim + r] = q_pe[b][h][r]                          (r < rope_dim)
 * BF16 in, FP32 accumulation, BF16 out: the decode's query [B, H, D + Dr] in the rotated
 * frame when w_kc has the read rotation folded in.  Replaces torch.bmm(q_nope, w_kc) and the
 * cat with q_pe of the DeepSeek MLA forward (deployment/patches/rolaq_sglang.patch:205-248,
 * with w_kc from fold_read_rotation, deployment/sglang/srt/mem_cache/rolaq_mla.py:56-71).
 *   q_nope  bf16 [B, H, nope_dim] with strides (qn_stride_b, qn_stride_h); nope_dim % 64 == 0
 *   w_kc    bf16 [H, latent_dim, nope_dim] contiguous (SGLang's storage of w_kc)
 *   q_pe    bf16 [B, H, rope_dim] or NULL when rope_dim == 0
 *   q_out   bf16 [B, H, latent_dim + rope_dim] with strides (q_stride_b, q_stride_h)
 */
int rolaq_absorb_query(const uint16_t* q_nope, int64_t qn_stride_b, int64_t qn_stride_h, const uint16_t* q_pe,
                       int64_t qp_stride_b, int64_t qp_stride_h, const uint16_t* w_kc, int32_t batch, int32_t heads,
                       int32_t nope_dim, int32_t latent_dim, int32_t rope_dim, uint16_t* q_out, int64_t q_stride_b,
                       int64_t q_stride_h, int32_t* err, cudaStream_t stream);

/*
 * Output projection after the MLA decode, on tcgen05: per request b and head h,
 *   out[b][h][v] = sum_e o[b][h][e] * w_vc[h][v][e]
 * BF16 in, FP32 accumulation, BF16 out; with the read rotation folded into w_vc the decode's
 * rotated-frame output needs no un-rotation.  Replaces torch.bmm(attn_output, w_vc)
 * (deployment/patches/rolaq_sglang.patch:261-274 with rolaq_mla.py:56-71).
 *   o     bf16 [B, H, latent_dim] with strides (o_stride_b, o_stride_h)
 *   w_vc  bf16 [H, v_dim, latent_dim] contiguous (SGLang's storage of w_vc); v_dim in
 *         {64, 128, 256, 512}
 *   out   bf16 [B, H, v_dim] with strides (out_stride_b, out_stride_h)
 */
int rolaq_project_output(const uint16_t* o, int64_t o_stride_b, int64_t o_stride_h, const uint16_t* w_vc,
                         int32_t batch, int32_t heads, int32_t latent_dim, int32_t v_dim, uint16_t* out,
                         int64_t out_stride_b, int64_t out_stride_h, int32_t* err, cudaStream_t stream);

/*
 * LSE merge of normalised partials: for each row r in [0, rows) and part p in
 * [0, n_parts): o = part_o + r*row_stride + p*part_stride (D floats),
 * lse = part_lse[r*lse_row_stride + p*lse_part_stride] (natural log, -inf = empty).
 * Writes out_bf16 / out_f32 [rows, D] (row stride ld_out) and out_lse [rows]; any
 * output pointer may be NULL.  Used inside one GPU and, for sequence-split decode,
 * after an NCCL all-gather of the per-rank partials.
 */
int rolaq_merge_partials(const float* part_o, int64_t row_stride, int64_t part_stride,
                         const float* part_lse, int64_t lse_row_stride, int64_t lse_part_stride,
                         int32_t n_parts, int64_t rows, int32_t latent_dim, uint16_t* out_bf16,
                         float* out_f32, int64_t ld_out, float* out_lse, cudaStream_t stream);

/*
 * Sequence-split exchange over NVLink peer memory (no counterpart in the reference, which
 * serves one GPU: deployment/serve.py:135-136; the merge is the split-KV LSE merge of
 * packed_mla_decode_gf_fwd, deployment/patches/rolaq_sglang.patch:98-111).  Each rank of a
 * sequence-split decode owns a receive buffer of rolaq_peer_recv_bytes bytes (allocated with
 * rolaq_device_alloc, zeroed, and mapped into every other rank with the CUDA IPC helpers)
 * and a zeroed int32 state[2] of its own.  Per decode, on every rank in the same order:
 *   rolaq_peer_merge_push  merges the rank's split partials (the part_o / part_lse scratch of
 *                          a token-range rolaq_packed_decode) in FP32 and writes the result
 *                          into every rank's receive buffer (peer_recv: device array of the
 *                          world buffer addresses as mapped in this process), then flags it;
 *   rolaq_peer_wait_merge  waits (bounded: ROLAQ_DEV_PEER_TIMEOUT after ~2 s) until every
 *                          rank's partial has arrived and LSE-merges them into out.
 * rows = batch * heads; latent_dim 256 or 512.  The state and flags live on the device, so
 * the two calls may be captured in a CUDA graph and replayed.
 */
int64_t rolaq_peer_recv_bytes(int32_t world, int64_t rows, int32_t latent_dim);
int rolaq_peer_merge_push(const float* part_o, const float* part_lse, int32_t n_parts, int64_t rows,
                          int32_t latent_dim, const uint64_t* peer_recv, int32_t world, int32_t rank,
                          int32_t* state, cudaStream_t stream);
int rolaq_peer_wait_merge(const float* recv, int32_t world, int64_t rows, int32_t latent_dim,
                          const int32_t* state, uint16_t* out_bf16, float* out_f32, float* out_lse,
                          int32_t* err, cudaStream_t stream);

/* Device buffers for the exchange (cudaMalloc of the current device, zero-filled before the
 * call returns; cudaFree) and their CUDA IPC mappings: a handle is ROLAQ_IPC_HANDLE_BYTES
 * opaque bytes. */
#define ROLAQ_IPC_HANDLE_BYTES 64
int rolaq_device_alloc(int64_t bytes, void** ptr);
int rolaq_device_free(void* ptr);
int rolaq_ipc_get_handle(const void* ptr, void* handle);
int rolaq_ipc_open(const void* handle, void** ptr);
int rolaq_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* ROLAQ_B200_H_ */
