// extern "C" entry points of librolaq_b200.so (declared in include/rolaq_b200.h).
// Every function validates its arguments on the host before launching, returns a
// status code, and records a message for rolaq_last_error() on failure.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kernels.cuh"

namespace rolaq {

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

}  // namespace rolaq

using namespace rolaq;

namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_cache(const rolaq_layer_cache* c, bool need_window, bool need_rope = true) {
  if (c == nullptr) return fail(ROLAQ_EINVAL, "cache is NULL");
  if (c->latent_dim != 256 && c->latent_dim != 512)
    return fail(ROLAQ_EUNSUPPORTED, "latent_dim %d unsupported (256 or 512)", c->latent_dim);
  if (need_rope && (c->rope_dim <= 0 || c->rope_dim % 16 != 0 || c->rope_dim > 128))
    return fail(ROLAQ_EUNSUPPORTED, "rope_dim %d unsupported (multiple of 16, <= 128)", c->rope_dim);
  if (!c->codes || !c->params || (need_rope && !c->rope))
    return fail(ROLAQ_EINVAL, "cache codes/params/rope must be non-NULL");
  if (!aligned16(c->codes) || !aligned16(c->params) || (need_rope && !aligned16(c->rope)))
    return fail(ROLAQ_EINVAL, "cache codes/params/rope must be 16-byte aligned");
  if (c->num_slots <= 0 || c->num_slots >= (int64_t(1) << 31))
    return fail(ROLAQ_EINVAL, "num_slots %lld out of range", (long long)c->num_slots);
  if (c->sink < 0 || c->recent < 0) return fail(ROLAQ_EINVAL, "sink/recent must be >= 0");
  if (need_window && c->sink + c->recent > 0) {
    if (!c->hp || !c->rows || !c->owners) return fail(ROLAQ_EINVAL, "window enabled but hp/rows/owners is NULL");
    if (!aligned16(c->hp)) return fail(ROLAQ_EINVAL, "hp must be 16-byte aligned");
    if (c->max_reqs < 0 || c->num_ring_rows < 1 + c->max_reqs * (c->sink + c->recent))
      return fail(ROLAQ_EINVAL, "num_ring_rows %lld < 1 + max_reqs*(sink+recent)", (long long)c->num_ring_rows);
  }
  return ROLAQ_OK;
}

int codec_ok(const rolaq_codec& k) {
  if (k.family == ROLAQ_CODEC_UNIFORM) return ROLAQ_OK;  // no scalars
  if (k.family != ROLAQ_CODEC_LLOYD) return fail(ROLAQ_EINVAL, "unknown codec family %d", (int)k.family);
  if (!(k.threshold > 0.f) || !(k.scale_factor > 0.f) || !(k.threshold < 1e30f) || !(k.scale_factor < 1e30f))
    return fail(ROLAQ_EINVAL, "codec threshold and scale_factor must be finite and > 0");
  return ROLAQ_OK;
}

int cuda_rc(int rc, const char* what) {
  if (rc == ROLAQ_ECUDA) {
    cudaError_t e = cudaGetLastError();
    return fail(ROLAQ_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return rc;
}

}  // namespace

extern "C" {

int rolaq_version(void) { return 10000; }

const char* rolaq_last_error(void) { return g_msg; }

int rolaq_check_device(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(ROLAQ_ECUDA, "no CUDA device");
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(ROLAQ_EUNSUPPORTED, "device is sm_%d%d; this library is built for sm_100a only", major, minor);
  if (encode_fn() == nullptr) return fail(ROLAQ_ECUDA, "cuTensorMapEncodeTiled unavailable");
  return ROLAQ_OK;
}

int rolaq_scatter_pack_rows(const float* x, int64_t ldx, const void* slots, int slots_are_int64, int64_t n,
                            int32_t latent_dim, int32_t group_size, rolaq_codec codec, uint8_t* codes,
                            float* params, int64_t num_slots, int32_t* err, cudaStream_t stream) {
  if (n < 0) return fail(ROLAQ_EINVAL, "n < 0");
  if (group_size != 128) return fail(ROLAQ_EUNSUPPORTED, "group_size %d unsupported (128)", group_size);
  if (latent_dim <= 0 || latent_dim % 128) return fail(ROLAQ_EUNSUPPORTED, "latent_dim must be a multiple of 128");
  if (n == 0) return ROLAQ_OK;
  if (!x || !slots || !codes || !params) return fail(ROLAQ_EINVAL, "NULL pointer");
  if (!aligned16(x) || ldx < latent_dim || ldx % 4) return fail(ROLAQ_EINVAL, "x must be 16-byte aligned, ldx >= D, ldx %% 4 == 0");
  if (!aligned16(codes) || !aligned16(params)) return fail(ROLAQ_EINVAL, "codes/params must be 16-byte aligned");
  if (int rc = codec_ok(codec)) return rc;
  return cuda_rc(launch_scatter_pack(x, ldx, slots, slots_are_int64, n, latent_dim, codec, codes, params, num_slots,
                                     err, stream),
                 "scatter_pack");
}

int rolaq_write_aux(const float* c, int64_t ldc, const uint16_t* k_pe, int64_t ld_pe, const int64_t* slots,
                    const void* seq_lens, int seq_lens_is64, const void* req_idx, int req_idx_is64,
                    const void* positions, int positions_is64, int64_t n, const rolaq_layer_cache* cache,
                    int32_t* err, cudaStream_t stream) {
  if (n < 0) return fail(ROLAQ_EINVAL, "n < 0");
  if (int rc = check_cache(cache, seq_lens != nullptr && req_idx != nullptr)) return rc;
  if (n == 0) return ROLAQ_OK;
  if (!c || !k_pe || !slots) return fail(ROLAQ_EINVAL, "NULL pointer");
  if (ldc < cache->latent_dim || ld_pe < cache->rope_dim) return fail(ROLAQ_EINVAL, "row stride too small");
  return cuda_rc(launch_aux(c, ldc, k_pe, ld_pe, slots, seq_lens, seq_lens_is64, req_idx, req_idx_is64, positions,
                            positions_is64, n, *cache, err, stream),
                 "write_aux");
}

int rolaq_fused_write(const uint16_t* c_kv, int64_t ld_ckv, const uint16_t* k_pe, int64_t ld_pe,
                      const int64_t* slots, const void* seq_lens, int seq_lens_is64, const void* req_idx,
                      int req_idx_is64, const void* positions, int positions_is64, int64_t n,
                      const uint16_t* rot_t, rolaq_codec codec, const rolaq_layer_cache* cache, int32_t* err,
                      cudaStream_t stream) {
  if (n < 0) return fail(ROLAQ_EINVAL, "n < 0");
  if (int rc = check_cache(cache, seq_lens != nullptr && req_idx != nullptr, k_pe != nullptr)) return rc;
  if (n == 0) return ROLAQ_OK;
  const int d = cache->latent_dim;
  if (!c_kv || !slots || !rot_t) return fail(ROLAQ_EINVAL, "NULL pointer");
  if (!aligned16(c_kv) || ld_ckv < d || ld_ckv % 8)
    return fail(ROLAQ_EINVAL, "c_kv must be 16-byte aligned with ld_ckv >= D and ld_ckv %% 8 == 0");
  if (k_pe && (!aligned16(k_pe) || ld_pe < cache->rope_dim || ld_pe % 8))
    return fail(ROLAQ_EINVAL, "k_pe must be 16-byte aligned with ld_pe >= Dr and ld_pe %% 8 == 0");
  if (!aligned16(rot_t)) return fail(ROLAQ_EINVAL, "rot_t must be 16-byte aligned");
  if (n >= (int64_t(1) << 31)) return fail(ROLAQ_EINVAL, "n too large");
  if (int rc = codec_ok(codec)) return rc;
  WriterArgs a{};
  a.n = n;
  a.d = d;
  a.k_pe = k_pe;
  a.ld_pe = ld_pe;
  a.slots = slots;
  a.seq_lens = seq_lens;
  a.seq_is64 = seq_lens_is64;
  a.req_idx = req_idx;
  a.req_is64 = req_idx_is64;
  a.positions = positions;
  a.pos_is64 = positions_is64;
  a.codec = codec;
  a.cache = *cache;
  a.err = err;
  return cuda_rc(launch_writer(c_kv, ld_ckv, rot_t, a, false, stream), "fused_write");
}

int rolaq_rotate_rows(const uint16_t* x, int64_t ldx, int64_t n, int32_t latent_dim, const uint16_t* w,
                      float* out_f32, uint16_t* out_bf16, int64_t ld_out, cudaStream_t stream) {
  if (n < 0) return fail(ROLAQ_EINVAL, "n < 0");
  if (latent_dim != 256 && latent_dim != 512)
    return fail(ROLAQ_EUNSUPPORTED, "latent_dim %d unsupported (256 or 512)", latent_dim);
  if (n == 0) return ROLAQ_OK;
  if (!x || !w || (!out_f32 && !out_bf16)) return fail(ROLAQ_EINVAL, "NULL pointer");
  if (!aligned16(x) || ldx < latent_dim || ldx % 8) return fail(ROLAQ_EINVAL, "x must be 16-byte aligned, ldx %% 8 == 0");
  if (!aligned16(w)) return fail(ROLAQ_EINVAL, "w must be 16-byte aligned");
  if (ld_out < latent_dim || ld_out % 8 || (out_f32 && !aligned16(out_f32)) || (out_bf16 && !aligned16(out_bf16)))
    return fail(ROLAQ_EINVAL, "outputs must be 16-byte aligned with ld_out %% 8 == 0");
  WriterArgs a{};
  a.n = n;
  a.d = latent_dim;
  a.out_f32 = out_f32;
  a.out_bf16 = out_bf16;
  a.ld_out = ld_out;
  return cuda_rc(launch_writer(x, ldx, w, a, true, stream), "rotate_rows");
}

int rolaq_dequant_rows(const uint8_t* codes, const float* params, const void* slots, int slots_are_int64, int64_t n,
                       int32_t latent_dim, int64_t num_slots, float* out_f32, uint16_t* out_bf16, int64_t ld_out,
                       int32_t* err, cudaStream_t stream) {
  if (n < 0) return fail(ROLAQ_EINVAL, "n < 0");
  if (latent_dim <= 0 || latent_dim % 128) return fail(ROLAQ_EUNSUPPORTED, "latent_dim must be a multiple of 128");
  if (n == 0) return ROLAQ_OK;
  if (!codes || !params || (!out_f32 && !out_bf16)) return fail(ROLAQ_EINVAL, "NULL pointer");
  if (ld_out < latent_dim || ld_out % 4 || (out_f32 && !aligned16(out_f32)) ||
      (out_bf16 && (reinterpret_cast<uintptr_t>(out_bf16) & 7)))
    return fail(ROLAQ_EINVAL, "outputs misaligned or ld_out too small");
  return cuda_rc(launch_dequant(codes, params, slots, slots_are_int64, n, latent_dim, num_slots, out_f32, out_bf16,
                                ld_out, err, stream),
                 "dequant_rows");
}

int rolaq_prepare_gf_splits(const int32_t* splits, int32_t* quant, int32_t* merge, int64_t n, cudaStream_t stream) {
  if (n < 0) return fail(ROLAQ_EINVAL, "n < 0");
  if (n == 0) return ROLAQ_OK;
  if (!splits || !quant || !merge) return fail(ROLAQ_EINVAL, "NULL pointer");
  return cuda_rc(launch_prepare_splits(splits, quant, merge, n, stream), "prepare_gf_splits");
}

int rolaq_packed_decode(const uint16_t* q, int64_t q_stride_b, int64_t q_stride_h, int32_t batch, int32_t heads,
                        const rolaq_layer_cache* cache, const int32_t* page_table, int64_t pt_stride,
                        int32_t max_pages, const int32_t* seq_lens, const int32_t* token_range, float sm_scale,
                        int32_t num_splits,
                        float* part_o, float* part_lse, uint16_t* out, int64_t out_stride_b, int64_t out_stride_h,
                        float* out_lse, int32_t* err, cudaStream_t stream) {
  if (batch < 0) return fail(ROLAQ_EINVAL, "batch < 0");
  if (int rc = check_cache(cache, true)) return rc;
  const int d = cache->latent_dim;
  if (!((d == 512 && cache->rope_dim == 64 && (heads == 16 || heads == 8)) ||
        (d == 256 && cache->rope_dim == 32 && (heads == 40 || heads == 16))))
    return fail(ROLAQ_EUNSUPPORTED, "decode shape D=%d Dr=%d H=%d not built (512/64/{8,16}, 256/32/{16,40})", d,
                cache->rope_dim, heads);
  if (cache->sink + cache->recent > 32) return fail(ROLAQ_EUNSUPPORTED, "sink + recent must be <= 32");
  if (num_splits < 1 || num_splits > 1024) return fail(ROLAQ_EINVAL, "num_splits must be in [1, 1024]");
  if (!(sm_scale > 0.f)) return fail(ROLAQ_EINVAL, "sm_scale must be > 0");
  if (batch == 0) return ROLAQ_OK;
  if (batch > 65535) return fail(ROLAQ_EINVAL, "batch must be <= 65535");
  if (!q || !page_table || !seq_lens || !part_o || !part_lse) return fail(ROLAQ_EINVAL, "NULL pointer");
  if (max_pages <= 0 || pt_stride < max_pages) return fail(ROLAQ_EINVAL, "page table shape");
  if (q_stride_h < d + cache->rope_dim || q_stride_b < heads * q_stride_h)
    return fail(ROLAQ_EINVAL, "q strides too small");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_stride_h & 1) || (q_stride_b & 1))
    return fail(ROLAQ_EINVAL, "q must be 4-byte aligned with even strides");
  if (out && (out_stride_h < d || out_stride_b < heads * out_stride_h))
    return fail(ROLAQ_EINVAL, "out strides too small");
  DecodeArgs a{};
  a.q = q;
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.batch = batch;
  a.cache = *cache;
  a.page_table = page_table;
  a.pt_stride = pt_stride;
  a.max_pages = max_pages;
  a.seq_lens = seq_lens;
  a.token_range = token_range;
  a.sm_scale = sm_scale;
  a.num_splits = num_splits;
  a.part_o = part_o;
  a.part_lse = part_lse;
  a.err = err;
  if (!out) return cuda_rc(launch_decode_partials(a, heads, stream), "packed_decode");  // the partials only
  {
    const int fused = launch_decode_merged(a, heads, out, out_stride_b, out_stride_h, out_lse, stream);
    if (fused != ROLAQ_EUNSUPPORTED) return cuda_rc(fused, "packed_decode");
  }
  int rc = cuda_rc(launch_decode(a, heads, stream), "packed_decode");
  if (rc != ROLAQ_OK) return rc;
  const int parts = num_splits + 1;
  // out rows are (b, h): row r = b * heads + h, at out + b*out_stride_b + h*out_stride_h
  if (out_stride_b == heads * out_stride_h) {
    return cuda_rc(launch_merge(part_o, int64_t(parts) * d, d, part_lse, parts, 1, parts, int64_t(batch) * heads, d,
                                out, nullptr, out_stride_h, out_lse, stream),
                   "merge");
  }
  for (int b = 0; b < batch; ++b) {
    rc = cuda_rc(launch_merge(part_o + int64_t(b) * heads * parts * d, int64_t(parts) * d, d,
                              part_lse + int64_t(b) * heads * parts, parts, 1, parts, heads, d,
                              out + int64_t(b) * out_stride_b, nullptr, out_stride_h,
                              out_lse ? out_lse + int64_t(b) * heads : nullptr, stream),
                 "merge");
    if (rc != ROLAQ_OK) return rc;
  }
  return ROLAQ_OK;
}

int64_t rolaq_peer_recv_bytes(int32_t world, int64_t rows, int32_t latent_dim) {
  if (world < 1 || rows < 0 || (latent_dim != 256 && latent_dim != 512)) return -1;
  return peer_recv_bytes(world, rows, latent_dim);
}

int rolaq_peer_merge_push(const float* part_o, const float* part_lse, int32_t n_parts, int64_t rows,
                          int32_t latent_dim, const uint64_t* peer_recv, int32_t world, int32_t rank, int32_t* state,
                          cudaStream_t stream) {
  if (latent_dim != 256 && latent_dim != 512) return fail(ROLAQ_EUNSUPPORTED, "latent_dim must be 256 or 512");
  if (world < 1 || world > 64 || rank < 0 || rank >= world) return fail(ROLAQ_EINVAL, "rank / world out of range");
  if (n_parts < 1 || rows < 0 || rows > (1 << 24)) return fail(ROLAQ_EINVAL, "n_parts < 1 or rows out of range");
  if (rows == 0) return ROLAQ_OK;
  if (!part_o || !part_lse || !peer_recv || !state) return fail(ROLAQ_EINVAL, "NULL pointer");
  if (reinterpret_cast<uintptr_t>(part_o) & 15) return fail(ROLAQ_EINVAL, "part_o must be 16-byte aligned");
  return cuda_rc(launch_peer_merge_push(part_o, part_lse, n_parts, static_cast<int>(rows), latent_dim, peer_recv, world,
                                        rank, state, stream),
                 "peer_merge_push");
}

int rolaq_peer_wait_merge(const float* recv, int32_t world, int64_t rows, int32_t latent_dim, const int32_t* state,
                          uint16_t* out_bf16, float* out_f32, float* out_lse, int32_t* err, cudaStream_t stream) {
  if (latent_dim != 256 && latent_dim != 512) return fail(ROLAQ_EUNSUPPORTED, "latent_dim must be 256 or 512");
  if (world < 1 || world > 64 || rows < 0 || rows > (1 << 24)) return fail(ROLAQ_EINVAL, "world / rows out of range");
  if (rows == 0) return ROLAQ_OK;
  if (!recv || !state) return fail(ROLAQ_EINVAL, "NULL pointer");
  if ((reinterpret_cast<uintptr_t>(recv) & 15) || (reinterpret_cast<uintptr_t>(out_bf16) & 15) ||
      (reinterpret_cast<uintptr_t>(out_f32) & 15))
    return fail(ROLAQ_EINVAL, "recv and outputs must be 16-byte aligned");
  return cuda_rc(launch_peer_wait_merge(recv, world, static_cast<int>(rows), latent_dim, state, out_bf16, out_f32,
                                        out_lse, err, stream),
                 "peer_wait_merge");
}

int rolaq_device_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes <= 0) return fail(ROLAQ_EINVAL, "bytes must be > 0 and ptr non-NULL");
  *ptr = nullptr;
  if (cudaMalloc(ptr, static_cast<size_t>(bytes)) != cudaSuccess) return cuda_rc(ROLAQ_ECUDA, "device_alloc");
  if (cudaMemset(*ptr, 0, static_cast<size_t>(bytes)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_rc(ROLAQ_ECUDA, "device_alloc");
  }
  return ROLAQ_OK;
}

int rolaq_device_free(void* ptr) {
  if (!ptr) return ROLAQ_OK;
  return cuda_rc(cudaFree(ptr) == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA, "device_free");
}

int rolaq_ipc_get_handle(const void* ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == ROLAQ_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle) return fail(ROLAQ_EINVAL, "NULL pointer");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return cuda_rc(ROLAQ_ECUDA, "ipc_get_handle");
  memcpy(handle, &h, sizeof(h));
  return ROLAQ_OK;
}

int rolaq_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(ROLAQ_EINVAL, "NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return cuda_rc(ROLAQ_ECUDA, "ipc_open");
  return ROLAQ_OK;
}

int rolaq_ipc_close(void* ptr) {
  if (!ptr) return ROLAQ_OK;
  return cuda_rc(cudaIpcCloseMemHandle(ptr) == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA, "ipc_close");
}

int rolaq_merge_partials(const float* part_o, int64_t row_stride, int64_t part_stride, const float* part_lse,
                         int64_t lse_row_stride, int64_t lse_part_stride, int32_t n_parts, int64_t rows,
                         int32_t latent_dim, uint16_t* out_bf16, float* out_f32, int64_t ld_out, float* out_lse,
                         cudaStream_t stream) {
  if (rows < 0 || n_parts < 1) return fail(ROLAQ_EINVAL, "rows < 0 or n_parts < 1");
  if (latent_dim <= 0) return fail(ROLAQ_EINVAL, "latent_dim <= 0");
  if (rows == 0) return ROLAQ_OK;
  if (!part_o || !part_lse) return fail(ROLAQ_EINVAL, "NULL pointer");
  if ((out_bf16 || out_f32) && ld_out < latent_dim) return fail(ROLAQ_EINVAL, "ld_out too small");
  if (rows > 0x7FFFFFFF) return fail(ROLAQ_EINVAL, "too many rows");
  return cuda_rc(launch_merge(part_o, row_stride, part_stride, part_lse, lse_row_stride, lse_part_stride, n_parts,
                              rows, latent_dim, out_bf16, out_f32, ld_out, out_lse, stream),
                 "merge");
}

int rolaq_page_table_from_req_to_token(const int32_t* req_to_token, int64_t rt_stride, const void* req_pool_indices,
                                       int req_is64, const void* seq_lens, int seq_lens_is64, int64_t batch,
                                       int32_t max_pages, int32_t* page_table, int64_t pt_stride,
                                       int32_t* seq_lens_out, int32_t* err, cudaStream_t stream) {
  if (batch < 0 || max_pages < 0) return fail(ROLAQ_EINVAL, "batch and max_pages must be >= 0");
  if (batch == 0 || max_pages == 0) return ROLAQ_OK;
  if (!req_to_token || !req_pool_indices || !seq_lens || !page_table)
    return fail(ROLAQ_EINVAL, "req_to_token, req_pool_indices, seq_lens and page_table must be non-NULL");
  if (rt_stride < int64_t(max_pages) * 64 || pt_stride < max_pages)
    return fail(ROLAQ_EINVAL, "req_to_token rows must hold max_pages * 64 tokens and page_table rows max_pages");
  if (batch > 65535) return fail(ROLAQ_EUNSUPPORTED, "batch %lld > 65535", (long long)batch);
  return cuda_rc(launch_page_table(req_to_token, rt_stride, req_pool_indices, req_is64, seq_lens, seq_lens_is64,
                                   batch, max_pages, page_table, pt_stride, seq_lens_out, err, stream),
                 "page_table_from_req_to_token");
}

int rolaq_absorb_query(const uint16_t* q_nope, int64_t qn_stride_b, int64_t qn_stride_h, const uint16_t* q_pe,
                       int64_t qp_stride_b, int64_t qp_stride_h, const uint16_t* w_kc, int32_t batch, int32_t heads,
                       int32_t nope_dim, int32_t latent_dim, int32_t rope_dim, uint16_t* q_out, int64_t q_stride_b,
                       int64_t q_stride_h, int32_t* err, cudaStream_t stream) {
  if (batch < 0 || heads <= 0) return fail(ROLAQ_EINVAL, "batch must be >= 0 and heads > 0");
  if (batch == 0) return ROLAQ_OK;
  if (!q_nope || !w_kc || !q_out) return fail(ROLAQ_EINVAL, "q_nope, w_kc and q_out must be non-NULL");
  if (nope_dim <= 0 || nope_dim % 64 != 0 || nope_dim > 1024)
    return fail(ROLAQ_EUNSUPPORTED, "nope_dim %d must be a positive multiple of 64 (<= 1024)", nope_dim);
  if (latent_dim != 256 && latent_dim != 512)
    return fail(ROLAQ_EUNSUPPORTED, "latent_dim %d unsupported (256 or 512)", latent_dim);
  if (rope_dim < 0 || rope_dim % 8 != 0 || (rope_dim > 0 && !q_pe))
    return fail(ROLAQ_EINVAL, "rope_dim must be a multiple of 8, with q_pe when > 0");
  if (!aligned16(q_nope) || !aligned16(w_kc) || !aligned16(q_out) || (q_pe && !aligned16(q_pe)))
    return fail(ROLAQ_EINVAL, "q_nope, q_pe, w_kc and q_out must be 16-byte aligned");
  if (qn_stride_b % 8 || qn_stride_h % 8 || q_stride_b % 8 || q_stride_h % 8 ||
      (rope_dim > 0 && (qp_stride_b % 8 || qp_stride_h % 8)))
    return fail(ROLAQ_EINVAL, "row strides must be multiples of 8 elements");
  ProjArgs a{q_nope, qn_stride_b, qn_stride_h, w_kc, q_out, q_stride_b, q_stride_h,
             rope_dim > 0 ? q_pe : nullptr, qp_stride_b, qp_stride_h, rope_dim, batch, heads, latent_dim, nope_dim, err};
  return cuda_rc(launch_proj(a, stream), "absorb_query");
}

int rolaq_project_output(const uint16_t* o, int64_t o_stride_b, int64_t o_stride_h, const uint16_t* w_vc,
                         int32_t batch, int32_t heads, int32_t latent_dim, int32_t v_dim, uint16_t* out,
                         int64_t out_stride_b, int64_t out_stride_h, int32_t* err, cudaStream_t stream) {
  if (batch < 0 || heads <= 0) return fail(ROLAQ_EINVAL, "batch must be >= 0 and heads > 0");
  if (batch == 0) return ROLAQ_OK;
  if (!o || !w_vc || !out) return fail(ROLAQ_EINVAL, "o, w_vc and out must be non-NULL");
  if (latent_dim != 256 && latent_dim != 512)
    return fail(ROLAQ_EUNSUPPORTED, "latent_dim %d unsupported (256 or 512)", latent_dim);
  if (v_dim != 64 && v_dim != 128 && v_dim != 256 && v_dim != 512)
    return fail(ROLAQ_EUNSUPPORTED, "v_dim %d unsupported (64, 128, 256 or 512)", v_dim);
  if (!aligned16(o) || !aligned16(w_vc) || !aligned16(out))
    return fail(ROLAQ_EINVAL, "o, w_vc and out must be 16-byte aligned");
  if (o_stride_b % 8 || o_stride_h % 8 || out_stride_b % 8 || out_stride_h % 8)
    return fail(ROLAQ_EINVAL, "row strides must be multiples of 8 elements");
  ProjArgs a{o, o_stride_b, o_stride_h, w_vc, out, out_stride_b, out_stride_h, nullptr, 0, 0, 0,
             batch, heads, v_dim, latent_dim, err};
  return cuda_rc(launch_proj(a, stream), "project_output");
}

}  // extern "C"

// ---- rolaq_packed_decode_static: the split partials in a fixed device array --------------------
// For callers that cannot allocate at decode time.  The scratch (part_o followed by part_lse,
// 32 MiB of FP32) is a file-scope device array of this library; its address is resolved once
// per device (the first call on a device, which should come before any stream capture) and
// cached.  Every element a call reads is written earlier in the same call, so nothing needs to
// start at zero; two calls that overlap in time on one device (any streams) share the array
// and race.
namespace {

constexpr int64_t kStaticPartFloats = int64_t(8) << 20;
__device__ __align__(256) float g_static_parts[kStaticPartFloats];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
float* g_static_ptr[kMaxDevices] = {};

int static_parts(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(ROLAQ_ECUDA, "no CUDA device");
  if (dev < 0 || dev >= kMaxDevices) return fail(ROLAQ_EUNSUPPORTED, "device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_parts);
    if (e != cudaSuccess) return fail(ROLAQ_ECUDA, "cudaGetSymbolAddress(static decode scratch): %s", cudaGetErrorString(e));
    g_static_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_static_ptr[dev];
  return ROLAQ_OK;
}

}  // namespace

extern "C" {

int64_t rolaq_packed_decode_static_capacity(void) { return kStaticPartFloats; }

int rolaq_packed_decode_static(const uint16_t* q, int64_t q_stride_b, int64_t q_stride_h, int32_t batch,
                               int32_t heads, const rolaq_layer_cache* cache, const int32_t* page_table,
                               int64_t pt_stride, int32_t max_pages, const int32_t* seq_lens,
                               const int32_t* token_range, float sm_scale, int32_t num_splits, uint16_t* out,
                               int64_t out_stride_b, int64_t out_stride_h, float* out_lse, int32_t* err,
                               cudaStream_t stream) {
  if (batch < 0 || heads <= 0 || num_splits < 1 || num_splits > 1024 || batch > 65535 || heads > 1024)
    return fail(ROLAQ_EINVAL, "batch, heads or num_splits out of range");
  if (cache == nullptr) return fail(ROLAQ_EINVAL, "cache is NULL");
  const int64_t d = cache->latent_dim;
  if (d <= 0 || d > 4096) return fail(ROLAQ_EINVAL, "latent_dim out of range");
  const int64_t rows = int64_t(batch) * heads * (num_splits + 1);
  const int64_t need = rows * d + rows;  // part_o [B, H, S+1, D] then part_lse [B, H, S+1]
  if (need > kStaticPartFloats)
    return fail(ROLAQ_EINVAL,
                "static decode scratch holds %lld floats; batch %d x heads %d x (num_splits + 1) %d x "
                "(latent_dim + 1) needs %lld (use rolaq_packed_decode with caller scratch)",
                (long long)kStaticPartFloats, batch, heads, num_splits + 1, (long long)need);
  if (batch == 0) return ROLAQ_OK;
  float* base = nullptr;
  if (int rc = static_parts(&base)) return rc;
  return rolaq_packed_decode(q, q_stride_b, q_stride_h, batch, heads, cache, page_table, pt_stride, max_pages,
                             seq_lens, token_range, sm_scale, num_splits, base, base + rows * d, out, out_stride_b,
                             out_stride_h, out_lse, err, stream);
}

}  // extern "C"
