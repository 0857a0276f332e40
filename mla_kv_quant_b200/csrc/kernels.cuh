// Argument blocks and launchers shared between the kernel translation units and
// the C ABI (abi.cu).  Internal to the library.
#pragma once

#include "common.cuh"

namespace rolaq {

// Fused writer / rotation GEMM (writer.cu).
struct WriterArgs {
  int64_t n;
  int32_t d;
  // codec mode
  const uint16_t* k_pe;
  int64_t ld_pe;
  const int64_t* slots;
  const void* seq_lens;
  int seq_is64;
  const void* req_idx;
  int req_is64;
  const void* positions;
  int pos_is64;
  rolaq_codec codec;
  rolaq_layer_cache cache;
  int32_t* err;
  // plain (rotation-only) mode
  float* out_f32;
  uint16_t* out_bf16;
  int64_t ld_out;
};

// Packed decode (decode.cu).
struct DecodeArgs {
  const uint16_t* q;
  int64_t q_sb, q_sh;
  int32_t batch;
  rolaq_layer_cache cache;
  const int32_t* page_table;
  int64_t pt_stride;
  int32_t max_pages;
  const int32_t* seq_lens;
  const int32_t* token_range;  // [B, 2] or nullptr
  float sm_scale;
  int32_t num_splits;
  float* part_o;
  float* part_lse;
  int32_t* err;
};

// Per-head projection GEMM around the decode (proj.cu): out[b, h, :n] = x[b, h, :k] w[h]^T,
// w[h] = [n, k] row-major; optionally out[b, h, n : n + dr] = pe[b, h, :dr].
struct ProjArgs {
  const uint16_t* x;
  int64_t x_sb, x_sh;
  const uint16_t* w;
  uint16_t* out;
  int64_t o_sb, o_sh;
  const uint16_t* pe;
  int64_t pe_sb, pe_sh;
  int32_t dr;
  int32_t batch, heads, n, k;
  int32_t* err;
};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// abi.cu
EncodeTiledFn encode_fn();
int sm_count();

// writer.cu
int launch_writer(const uint16_t* x, int64_t ldx, const uint16_t* w, const WriterArgs& args, bool plain,
                  cudaStream_t stream);

// codec.cu
int launch_scatter_pack(const float* x, int64_t ldx, const void* slots, int slots64, int64_t n, int d,
                        rolaq_codec codec, uint8_t* codes, float* params, int64_t num_slots, int32_t* err,
                        cudaStream_t s);
int launch_aux(const float* c, int64_t ldc, const uint16_t* k_pe, int64_t ld_pe, const int64_t* slots,
               const void* seq, int seq64, const void* req, int req64, const void* pos, int pos64, int64_t n,
               const rolaq_layer_cache& cache, int32_t* err, cudaStream_t s);
int launch_dequant(const uint8_t* codes, const float* params, const void* slots, int slots64, int64_t n, int d,
                   int64_t num_slots, float* out_f32, uint16_t* out_bf16, int64_t ld_out, int32_t* err,
                   cudaStream_t s);
int launch_prepare_splits(const int32_t* splits, int32_t* quant, int32_t* merge, int64_t n, cudaStream_t s);

int launch_page_table(const int32_t* req_to_token, int64_t rt_stride, const void* req_idx, int req64,
                      const void* seq_lens, int seq64, int64_t batch, int32_t max_pages, int32_t* page_table,
                      int64_t pt_stride, int32_t* seq_out, int32_t* err, cudaStream_t s);

// proj.cu
int launch_proj(const ProjArgs& a, cudaStream_t s);

// decode.cu
int launch_decode(const DecodeArgs& a, int heads, cudaStream_t s);
// INT2 splits and the window/merge in one go where the fused kernels apply (D/Dr/H =
// 512/64/16, aligned output); ROLAQ_EUNSUPPORTED otherwise (nothing launched).
int launch_decode_merged(const DecodeArgs& a, int heads, uint16_t* out, int64_t out_sb, int64_t out_sh,
                         float* out_lse, cudaStream_t s);
int64_t peer_recv_bytes(int world, int64_t rows, int d);
int launch_decode_partials(const DecodeArgs& a, int heads, cudaStream_t s);
int launch_peer_merge_push(const float* part_o, const float* part_lse, int n_parts, int rows, int d,
                           const uint64_t* peers, int world, int rank, int32_t* state, cudaStream_t s);
int launch_peer_wait_merge(const float* recv, int world, int rows, int d, const int32_t* state, uint16_t* out_bf16,
                           float* out_f32, float* out_lse, int32_t* err, cudaStream_t s);
int launch_merge(const float* part_o, int64_t row_stride, int64_t part_stride, const float* part_lse,
                 int64_t lse_row_stride, int64_t lse_part_stride, int n_parts, int64_t rows, int d,
                 uint16_t* out_bf16, float* out_f32, int64_t ld_out, float* out_lse, cudaStream_t s);

}  // namespace rolaq
