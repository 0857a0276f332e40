// Sequence-split exchange over NVLink peer memory.
//
// Reference behaviour: the reference serves one GPU (deployment/serve.py:135-136); a long
// request split over ranks needs its (m, l, o) partials merged by log-sum-exp, the same merge
// as the split-KV merge of packed_mla_decode_gf_fwd (deployment/patches/rolaq_sglang.patch:98-111).
//
// Instead of a library all-gather, the kernel that merges a rank's splits writes the rank's
// FP32 slice partial straight into every rank's receive buffer (CUDA IPC mappings of one
// allocation per rank), and the final merge waits for every rank's partial:
//
//   merge_push_kernel  (rank r: its splits -> (o, lse) in FP32 -> recv[q][parity][r] for every q,
//                       then, by the grid's last CTA, flags_q[r] = step after a system fence)
//   wait_merge_kernel  (rank q: waits, bounded, until flags_q[r] >= step for every r, then merges
//                       recv[q][parity][0 .. world) -> BF16 / FP32 out)
//
// Receive buffer of a rank: float data[2][world][rows][D + 4] (step parity, source rank, row:
// o[D], lse, 3 pad floats), then int32 flags[world] (16-byte aligned).  A rank's own state
// (local memory): int32 [0] exchanges completed, [1] CTAs of the running push that finished.
// Double buffering by step parity suffices: a rank pushes step s + 2 only after its wait for
// step s + 1, which needs every rank's push of step s + 1, issued after that rank's merge of s.
#include "kernels.cuh"
#include "merge.cuh"

namespace rolaq {
namespace peer {

constexpr int kRowsPerCta = 4;

__device__ __forceinline__ void st_relaxed_sys(int32_t* p, int32_t v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// LSE merge of n partials of one row: o_k at o + k * o_stride (8 elements from column j), lse
// at lse[k * lse_stride].  Every lane of the warp handles the row (D / 8 threads per row, a
// multiple of 32); returns the merged 8 values (FP32) and the merged lse.  Lane k % 32 holds
// the weight of partial k; the partials' loads are issued eight at a time before any is used.
__device__ __forceinline__ float merge_row(const float* o, int64_t o_stride, const float* lse, int64_t lse_stride,
                                           int n, int lane, float (&acc)[8]) {
  float m = -INFINITY;
  for (int k = lane; k < n; k += 32) m = fmaxf(m, lse[k * lse_stride]);
  m = warp_max(m);
  const float mref = m == -INFINITY ? 0.f : m;
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.f;
  float den = 0.f;
  for (int k0 = 0; k0 < n; k0 += 32) {
    const int cnt = min(32, n - k0);
    const float lv = lane < cnt ? lse[(k0 + lane) * lse_stride] : -INFINITY;
    const float wl = lv != -INFINITY ? __expf(lv - mref) : 0.f;  // weight of partial k0 + lane
    den += wl;
    for (int q = 0; q < cnt; q += 8) {
      float4 v[8][2];
      float w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        w[u] = __shfl_sync(0xFFFFFFFFu, wl, (q + u) & 31);
        if (q + u >= cnt) w[u] = 0.f;
        const float4* src = reinterpret_cast<const float4*>(o + (k0 + min(q + u, cnt - 1)) * o_stride);
        v[u][0] = src[0];
        v[u][1] = src[1];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {  // empty partials (weight 0) are masked, not multiplied
        const float vv[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w, v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = w[u] > 0.f ? fmaf(w[u], vv[c], acc[c]) : acc[c];
      }
    }
  }
  den = warp_sum(den);
  const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] *= inv;
  return den > 0.f ? mref + logf(den) : -INFINITY;
}

// WIDE (many partials): a CTA per (row, 128-column chunk), its warps taking the partials in
// turn (wide::merge_chunk); else kRowsPerCta rows per CTA, D / 8 threads per row.
template <int D, bool WIDE>
__global__ void __launch_bounds__(WIDE ? wide::kThreads : kRowsPerCta * D / 8)
    merge_push_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int n_parts, int rows,
                      const uint64_t* __restrict__ peers, int world, int rank, int32_t* state) {
  constexpr int TPR = D / 8;  // threads per row
  const int64_t slot = int64_t(rows) * (D + 4);
  // launched as a programmatic dependent of the decode kernel: its partials (and, through it,
  // the window split's) are complete once this returns
  grid_dependency_wait();
  if (threadIdx.x == 0) grid_launch_dependents();  // the wait kernel may take its SMs now
  const int32_t step = state[0] + 1;  // this exchange; state[0] moves only when the whole grid is done
  if (WIDE) {
    __shared__ float4 red[wide::kWarps][32];
    constexpr int CH = D / wide::kCols;
    const int row = blockIdx.x / CH, c0 = (blockIdx.x % CH) * wide::kCols;
    float4 res;
    const float lse = wide::merge_chunk(part_o + int64_t(row) * n_parts * D, D, part_lse + int64_t(row) * n_parts, 1,
                                        n_parts, c0, D, red, res);
    if (threadIdx.x < 32) {
      const int64_t off = (int64_t(step & 1) * world + rank) * slot + int64_t(row) * (D + 4);
      for (int q = 0; q < world; ++q) {  // NVLink stores into every rank's receive buffer
        float* dst = reinterpret_cast<float*>(peers[q]) + off;
        reinterpret_cast<float4*>(dst + c0)[threadIdx.x] = res;
        if (c0 == 0 && threadIdx.x == 0) dst[D] = lse;
      }
    }
  } else {
    const int row = blockIdx.x * kRowsPerCta + threadIdx.x / TPR;
    const int j = 8 * (threadIdx.x % TPR), lane = threadIdx.x & 31;
    if (row < rows) {
      float acc[8];
      const float lse = merge_row(part_o + int64_t(row) * n_parts * D + j, D, part_lse + int64_t(row) * n_parts, 1,
                                  n_parts, lane, acc);
      const int64_t off = (int64_t(step & 1) * world + rank) * slot + int64_t(row) * (D + 4);
      for (int q = 0; q < world; ++q) {  // NVLink stores into every rank's receive buffer
        float* dst = reinterpret_cast<float*>(peers[q]) + off;
        reinterpret_cast<float4*>(dst + j)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        reinterpret_cast<float4*>(dst + j)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        if (j == 0) dst[D] = lse;
      }
    }
  }
  // The CTA's stores are ordered before its count by the barrier and a GPU-scope fence (every
  // CTA of the grid is on this GPU); the last CTA to count acquires them all and makes them
  // visible system-wide with one fence before it writes the flags.  That fence and each
  // flag store after it form a release pattern (a fence, then a strong store), and release
  // and acquire are cumulative, so a peer that acquires a flag sees every CTA's stores.  The
  // flag stores are relaxed: a release store would fence again, waiting for the previous
  // flag's NVLink round trip, so the world's flags would go out one round trip apart.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int done = atomicAdd(&state[1], 1);
    if (done == gridDim.x - 1) {  // the grid's last CTA
      __threadfence_system();
      for (int q = 0; q < world; ++q) {
        int32_t* flags = reinterpret_cast<int32_t*>(reinterpret_cast<float*>(peers[q]) + 2 * world * slot);
        st_relaxed_sys(flags + rank, step);
      }
      state[1] = 0;
      state[0] = step;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(kRowsPerCta * D / 8) wait_merge_kernel(const float* __restrict__ recv, int world,
                                                                        int rows, const int32_t* state,
                                                                        uint16_t* __restrict__ out_bf16,
                                                                        float* __restrict__ out_f32,
                                                                        float* __restrict__ out_lse, int32_t* err) {
  constexpr int TPR = D / 8;
  __shared__ int ok_all;
  const int64_t slot = int64_t(rows) * (D + 4);
  grid_dependency_wait();  // a programmatic dependent of this rank's push: state[0] is its step
  const int32_t step = state[0];
  if (threadIdx.x == 0) {
    const int32_t* flags = reinterpret_cast<const int32_t*>(recv + 2 * world * slot);
    bool ok = true;
    const uint64_t t0 = global_ns();
    for (int q = 0; q < world && ok; ++q) {
      uint32_t polls = 0;
      while (ld_acquire_sys(flags + q) < step) {  // bounded: a rank that never pushes ends the wait
        if ((++polls & 1023u) == 0 && (global_ns() - t0 > kWaitNs || polls >= kWaitPolls)) {
          ok = false;
          break;
        }
      }
    }
    if (!ok) report(err, ROLAQ_DEV_PEER_TIMEOUT);
    ok_all = ok;
  }
  __syncthreads();
  const int row = blockIdx.x * kRowsPerCta + threadIdx.x / TPR;
  const int j = 8 * (threadIdx.x % TPR), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float acc[8];
  const float* base = recv + int64_t(step & 1) * world * slot + int64_t(row) * (D + 4);
  float lse = -INFINITY;
  if (ok_all) {
    lse = merge_row(base + j, slot, base + D, slot, world, lane, acc);
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.f;
  }
  if (out_bf16) {
    uint32_t pk[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const __nv_bfloat162 v2 = __floats2bfloat162_rn(acc[2 * c], acc[2 * c + 1]);
      pk[c] = *reinterpret_cast<const uint32_t*>(&v2);
    }
    reinterpret_cast<uint4*>(out_bf16 + int64_t(row) * D + j)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  if (out_f32) {
    reinterpret_cast<float4*>(out_f32 + int64_t(row) * D + j)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    reinterpret_cast<float4*>(out_f32 + int64_t(row) * D + j)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  if (out_lse && j == 0) out_lse[row] = lse;
}

}  // namespace peer

int64_t peer_recv_bytes(int world, int64_t rows, int d) {
  return (2 * int64_t(world) * rows * (d + 4)) * 4 + ((int64_t(world) * 4 + 15) / 16) * 16;
}

// Both kernels are launched as programmatic dependents of the kernel before them in the stream
// (the decode kernel, then the push): their CTAs are placed while that grid runs and wait for
// its completion (griddepcontrol.wait) before reading what it wrote.
template <typename... KArgs, typename... Args>
static int launch_dependent(void (*kernel)(KArgs...), int ctas, int threads, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, args...) != cudaSuccess) return ROLAQ_ECUDA;
  return cudaGetLastError() == cudaSuccess ? ROLAQ_OK : ROLAQ_ECUDA;
}

int launch_peer_merge_push(const float* part_o, const float* part_lse, int n_parts, int rows, int d,
                           const uint64_t* peers, int world, int rank, int32_t* state, cudaStream_t s) {
  if (n_parts >= wide::kMinParts) {  // same rule as launch_merge, so both exchanges merge alike
    const int ctas = rows * (d / wide::kCols);
    if (d == 512)
      return launch_dependent(peer::merge_push_kernel<512, true>, ctas, wide::kThreads, s, part_o, part_lse, n_parts,
                              rows, peers, world, rank, state);
    return launch_dependent(peer::merge_push_kernel<256, true>, ctas, wide::kThreads, s, part_o, part_lse, n_parts,
                            rows, peers, world, rank, state);
  }
  const int ctas = (rows + peer::kRowsPerCta - 1) / peer::kRowsPerCta;
  if (d == 512)
    return launch_dependent(peer::merge_push_kernel<512, false>, ctas, peer::kRowsPerCta * 64, s, part_o, part_lse,
                            n_parts, rows, peers, world, rank, state);
  return launch_dependent(peer::merge_push_kernel<256, false>, ctas, peer::kRowsPerCta * 32, s, part_o, part_lse,
                          n_parts, rows, peers, world, rank, state);
}

int launch_peer_wait_merge(const float* recv, int world, int rows, int d, const int32_t* state, uint16_t* out_bf16,
                           float* out_f32, float* out_lse, int32_t* err, cudaStream_t s) {
  const int ctas = (rows + peer::kRowsPerCta - 1) / peer::kRowsPerCta;
  if (d == 512)
    return launch_dependent(peer::wait_merge_kernel<512>, ctas, peer::kRowsPerCta * 64, s, recv, world, rows, state,
                            out_bf16, out_f32, out_lse, err);
  return launch_dependent(peer::wait_merge_kernel<256>, ctas, peer::kRowsPerCta * 32, s, recv, world, rows, state,
                          out_bf16, out_f32, out_lse, err);
}

}  // namespace rolaq
