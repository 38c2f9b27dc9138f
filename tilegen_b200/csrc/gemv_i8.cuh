// Few-row INT8 GEMM ("GEMV") with the dequantising epilogue (sm_100a), for
// M <= 4 activation rows:
//
//   out[m,n] = ((float(sum_k xq[m,k]*wq[n,k]) * xscale[m]) * wscale[n]) + bias[n]
//
// the arithmetic of tilegen/quant/int8_ops.py:22-70, as in gemm_i8.cuh.  With
// one to four rows the product is a stream of the weight (N*K bytes, read
// once) with one to four multiply-adds per weight byte.  Tensor-core tiles
// would idle on it, and the split-K kernel's fixed latencies (TMEM allocation,
// the MMA pipeline, the cluster reduction) are a large part of a ~12 us
// stream.  Here the CUDA cores do it:
//  * a warp owns R = 4 consecutive weight rows over one part of K.  Lane l
//    reads the 16-byte chunks l, l + 32, ... of the four rows (128-bit loads
//    that skip L1) and the same chunks of the M activation rows (L1-cached:
//    every warp of the SM reads the same activations), and accumulates the
//    exact int32 dot products with dp4a (four signed byte products a step);
//  * K is split into KP = 1, 2, 4 or 8 parts so that a narrow weight still
//    puts enough warps on the stream; the parts of a row group are warps of
//    one CTA and their int32 partials meet in shared memory;
//  * before the programmatic-dependent wait each warp asks L2 for the first
//    quarter of its weight rows (cp.async.bulk.prefetch.L2), so the weight
//    stream starts while the activation quantiser launched before it runs.
//    A quarter: prefetching everything queues the whole weight ahead of the
//    loads that follow the wait (measured on B200, M = 1: a quarter gave the
//    fastest quantiser + GEMV pair, and a GEMV launched alone as fast as with
//    no prefetch).  Only L2: it is the point of coherence, so a line fetched
//    early is never stale, even if the kernel before wrote the weight.
// Integer sums are exact and order-independent, so the output is bit-identical
// to the tiled and split-K kernels and to the reference's torch sequence.
#pragma once

#include "common.cuh"

namespace tg {

namespace gemv {
constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr int R = 4;       // weight rows per warp
constexpr int M_MAX = 4;   // activation rows
// 16-byte chunks per lane in flight per row: two for one or two activation
// rows, one for four (register budget of 64 at four CTAs per SM).
__host__ __device__ constexpr int unroll(int mr) { return mr <= 2 ? 2 : 1; }
}  // namespace gemv

struct GemvParams {
  const int8_t* xq;
  const float* xscale;
  const int8_t* wq;
  const float* wscale;
  const void* bias;
  int bias_dtype;
  int wscale_bcast;
  int M, N, K;
  int kp;               // K parts per row group = warps per group (1, 2, 4 or 8)
  int part_chunks;      // 16-byte chunks of K per part
  int prefetch;         // 1: prefetch a quarter of each warp's weight rows into L2 first
  void* out;            // [M, N] of OUT
};

// 128-bit load of weight bytes read exactly once: not kept in L1, and L2
// fetches 256 bytes at a time (a warp reads 512 contiguous bytes of a row).
__device__ __forceinline__ int4 ld_stream_v4(const int4* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Bring `bytes` (a multiple of 16) at a 16-byte aligned address into L2.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ int32_t dp4a_v4(const int4 a, const int4 b, int32_t c) {
  c = __dp4a(a.x, b.x, c);
  c = __dp4a(a.y, b.y, c);
  c = __dp4a(a.z, b.z, c);
  return __dp4a(a.w, b.w, c);
}

// MR: activation rows the kernel is compiled for (p.M <= MR; the rows from
// p.M up read as zero and are not stored); OUT: tg_dtype.
template <int MR, int OUT, bool HAS_BIAS>
__global__ void __launch_bounds__(gemv::THREADS, 4) gemv_i8_kernel(const GemvParams p) {
  using namespace gemv;
  constexpr int U = unroll(MR);
  constexpr int RM = R * MR;
  __shared__ int32_t partial[WARPS][RM];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kp = p.kp;
  const int groups_per_cta = WARPS / kp;
  const int g_local = warp / kp;
  const int part = warp - g_local * kp;
  const int n0 = (blockIdx.x * groups_per_cta + g_local) * R;
  const int nch = p.K >> 4;
  const int c0 = part * p.part_chunks;
  const int c1 = min(c0 + p.part_chunks, nch);
  // N is a multiple of 4 (16-byte output rows), so a group is whole or absent.
  const bool live = n0 < p.N && c0 < c1;

  if (live && p.prefetch && lane < R)
    prefetch_l2_bulk(p.wq + (size_t(n0 + lane) * size_t(nch) + size_t(c0)) * 16u, uint32_t(c1 - c0 + 3) / 4u * 16u);
  // Wait for the kernel that wrote xq / xscale (the activation quantiser).
  pdl_wait();

  int32_t acc[R][MR];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0;

  if (live) {
    const int4* w = reinterpret_cast<const int4*>(p.wq) + size_t(n0) * size_t(nch);
    const int4* x = reinterpret_cast<const int4*>(p.xq);
    const int M = p.M;
#pragma unroll 1
    for (int c = c0 + lane; c < c1; c += 32 * U) {
      int4 wv[U][R];
      int4 xv[U][MR];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cc = c + 32 * u;
        const bool in = cc < c1;
#pragma unroll
        for (int r = 0; r < R; ++r)
          wv[u][r] = in ? ld_stream_v4(w + size_t(r) * size_t(nch) + cc) : make_int4(0, 0, 0, 0);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          xv[u][m] = (in && m < M) ? __ldg(x + size_t(m) * size_t(nch) + cc) : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < MR; ++m) acc[r][m] = dp4a_v4(wv[u][r], xv[u][m], acc[r][m]);
    }
  }

  // Sum over the warp's lanes, then over the K parts of each row group.
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const int32_t s = __reduce_add_sync(0xffffffffu, acc[r][m]);
      if (lane == r * MR + m) partial[warp][r * MR + m] = s;
    }
  __syncthreads();

  const int t = threadIdx.x;
  if (t < groups_per_cta * RM) {
    const int g = t / RM;
    const int rm = t - g * RM;
    const int r = rm / MR;
    const int m = rm - r * MR;
    const int n = (blockIdx.x * groups_per_cta + g) * R + r;
    if (m < p.M && n < p.N) {
      int32_t sum = 0;
      for (int k = 0; k < kp; ++k) sum += partial[g * kp + k][rm];
      const float ws = p.wscale[p.wscale_bcast ? 0 : n];
      float bs = 0.0f;
      if (HAS_BIAS) {
        if (p.bias_dtype == TG_DT_F32) bs = static_cast<const float*>(p.bias)[n];
        else if (p.bias_dtype == TG_DT_F16) bs = __half2float(static_cast<const __half*>(p.bias)[n]);
        else bs = __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
      }
      char* o = static_cast<char*>(p.out) + (size_t(m) * size_t(p.N) + size_t(n)) * (OUT == 0 ? 4 : 2);
      store_dequant<OUT, HAS_BIAS>(o, sum, p.xscale[m], ws, bs);
    }
  }
}

}  // namespace tg
