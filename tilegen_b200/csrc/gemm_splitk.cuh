// Small-M INT8 GEMM with the dequantising epilogue (sm_100a), for M <= 128
// activation rows (decode / preview steps):
//
//   out[m,n] = ((float(sum_k xq[m,k]*wq[n,k]) * xscale[m]) * wscale[n]) + bias[n]
//
// the arithmetic of tilegen/quant/int8_ops.py:22-70, as in gemm_i8.cuh.  With
// few rows the work is streaming the weight (N*K bytes) once; the 128-row
// tiles of gemm_i8.cuh would put only N/256 CTAs on that stream.  Here:
//  * The roles of the operands are swapped: a 128-row tile of the WEIGHT is
//    the UMMA M operand and the (zero-padded) activation rows are UMMA N
//    (MPAD = 16, 32, 64 or 128), so D[n, m] accumulates in a 128-lane x MPAD-column
//    TMEM tile (tcgen05 kind::i8, int32).
//  * K is split: CTA (s, t) multiplies column tile t over k-blocks
//    [s*kb_per_slice, ...), so that N/128 x slices CTAs stream the weight
//    from all SMs.  Each CTA pulls its weight slice into L2 at start-up,
//    before the programmatic-dependent wait, so that stream overlaps the
//    activation quantiser launched before it.
//  * The partial tiles are summed in one of two ways (integer addition: exact
//    and order-independent either way), then dequantised with one rounding
//    per operation, as the reference:
//    - CL (K split at most 8 ways): the slices of a column tile are one
//      thread-block cluster.  Each CTA puts its partial tile in its own shared
//      memory (the finished operand ring); after a cluster barrier, CTA r
//      sums rows r, r + slices, ... from all of them over distributed shared
//      memory and stores them.  No scratch in global memory.
//    - otherwise each CTA adds its partial into an [M, N] int32 scratch
//      accumulator with red.global.add, then counts itself in count[t]; the
//      CTA that brings count[t] to `slices` reads the finished sums, stores
//      the output and writes zeros back over its accumulator tile and
//      counter.  That scratch is all-zero between launches (zero before the
//      first).
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2-5 epilogue.  Every wait is bounded (common.cuh).
#pragma once

#include "common.cuh"
#include "gemm_i8.cuh"

namespace tg {

namespace splitk {
constexpr int BNW = 128;                 // weight rows per tile (UMMA M)
constexpr int BK = 128;                  // bytes of K per k-block
constexpr int UK = 32;                   // K per tcgen05.mma kind::i8
constexpr uint32_t W_BYTES = BNW * BK;   // 16 KB
constexpr int THREADS = 192;
constexpr int M_MAX = 128;
// Ring depth: 4 slots, 3 when the activation tile is 128 rows (two CTAs per SM).
__host__ __device__ constexpr int stages(int mpad) { return mpad <= 64 ? 4 : 3; }
__host__ __device__ constexpr uint32_t x_bytes(int mpad) { return uint32_t(mpad) * BK; }
__host__ __device__ constexpr uint32_t stage_bytes(int mpad) { return W_BYTES + x_bytes(mpad); }
__host__ __device__ constexpr uint32_t smem_bytes(int mpad) { return stages(mpad) * stage_bytes(mpad) + 1024; }
}  // namespace splitk

struct SplitKParams {
  const float* xscale;
  const float* wscale;
  const void* bias;
  int bias_dtype;
  int wscale_bcast;
  int M, N, K;
  int k_blocks;      // ceil(K / 128)
  int kb_per_slice;  // k-blocks per CTA
  int slices;        // CTAs per column tile (gridDim.x)
  int32_t* acc;      // [M, N] partial sums: zero on entry, zero on exit
  uint32_t* count;   // [ceil(N / 128)] finished slices: zero on entry, zero on exit
  void* out;         // [M, N] of OUT
};

// MPAD: activation rows padded to 16, 32, 64 or 128 (the UMMA N); OUT: tg_dtype;
// CL: launched with clusters of gridDim.x CTAs (all slices of a column tile).
template <int MPAD, int OUT, bool HAS_BIAS, bool CL>
__global__ void __launch_bounds__(splitk::THREADS, 1)
    gemm_i8_splitk_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x,
                          const SplitKParams p) {
  using namespace splitk;
  static_assert(MPAD % 16 == 0 && MPAD >= 16 && MPAD <= M_MAX, "padded rows");
  constexpr uint32_t XB = x_bytes(MPAD);
  constexpr uint32_t TX_BYTES = W_BYTES + XB;
  constexpr int STAGES = stages(MPAD);
  constexpr uint32_t TMEM_COLS = MPAD <= 32 ? 32 : (MPAD <= 64 ? 64 : 128);
  constexpr uint32_t IDESC = gemm::idesc(BNW, MPAD);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * W_BYTES;

  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ int last_slice;
  __shared__ int issued;  // TMA loads the producer issued

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int slice = blockIdx.x;
  const int tile = blockIdx.y;
  const int n0 = tile * BNW;
  const int kb0 = slice * p.kb_per_slice;
  const int kb1 = min(kb0 + p.kb_per_slice, p.k_blocks);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tma_w);
    prefetch_tmap(&tma_x);
    // The weight stream is this kernel's whole cost at small M and does not
    // depend on the kernel before it: pull this CTA's slice of W into L2 now,
    // while that kernel (the activation quantiser) may still be running, so
    // the loads after the programmatic-dependent wait hit L2.  Only into L2:
    // the weights may have been written by the kernel before, so nothing lands
    // in shared memory until that wait.
    for (int kb = kb0; kb < kb1; ++kb) tma_prefetch_l2_2d(&tma_w, kb * BK, n0);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tfull_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
    issued = 0;
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  // Overlaps the end of the kernel that produced xq/xscale when launched as
  // its programmatic dependent; nothing below reads them before it completed.
  pdl_wait();

  auto wait = [&](uint64_t* bar, uint32_t parity, unsigned int err) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
      for (int i = 0; i < 32; ++i)
        if (mbar_try_wait(bar, parity)) return true;
      if (abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(&g_device_status, err);
        abort_flag = 1;
        return false;
      }
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int n_issued = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait(&empty_bar[stage], phase ^ 1u, DEVERR_PIPE_TIMEOUT)) break;
        mbar_arrive_expect_tx(&full_bar[stage], TX_BYTES);
        tma_load_2d(sW + stage * W_BYTES, &tma_w, &full_bar[stage], kb * BK, n0);
        tma_load_2d(sX + stage * XB, &tma_x, &full_bar[stage], kb * BK, 0);
        ++n_issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      issued = n_issued;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait(&full_bar[stage], phase, DEVERR_TMA_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t w_addr = smem_u32(sW + stage * W_BYTES);
        const uint32_t x_addr = smem_u32(sX + stage * XB);
#pragma unroll
        for (int k = 0; k < BK / UK; ++k)
          mma_i8(tmem_base, gemm::kmajor_sw128_desc(w_addr + k * UK), gemm::kmajor_sw128_desc(x_addr + k * UK),
                 IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
        mma_commit(&empty_bar[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) mma_commit(&tfull_bar);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 64;  // 0..127
    const int quarter = warp & 3;     // TMEM lanes [32*quarter, +32)
    const int n = n0 + quarter * 32 + lane;
    // Warp-uniform: tcgen05.ld below is executed by all 32 lanes or none.
    const bool got = __all_sync(0xffffffffu, wait(&tfull_bar, 0u, DEVERR_MMA_TIMEOUT));
    if (CL) {
      // The partial tile into this CTA's operand ring, which every MMA has
      // finished reading once tfull completed: P[m][nl], 128 int32 per row m,
      // consecutive lanes at consecutive words.
      int32_t* P = reinterpret_cast<int32_t*>(smem) + quarter * 32 + lane;
      if (got) {
        tc_fence_after();
#pragma unroll 1
        for (int h = 0; h < MPAD; h += 16) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(h), v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) P[(h + j) * BNW] = static_cast<int32_t>(v[j]);
        }
      }
    } else if (got) {
      tc_fence_after();
      // 16 columns (activation rows) at a time; coalesced over the warp: 32
      // consecutive n of one row m per add.
      int32_t* a = p.acc + n;
      const size_t stride = size_t(p.N);
#pragma unroll 1
      for (int h = 0; h < MPAD; h += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(h), v);
        tmem_wait_ld();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (h + j < p.M) atomicAdd(a + j * stride, static_cast<int32_t>(v[j]));
        }
        a += 16 * stride;
      }
      __threadfence();
    }
    if (!CL) {
      named_barrier(1, 128);
      // Counted even after a wait gave up (that slice then adds nothing), so
      // the last slice still returns the scratch to zero; the status word
      // reports the failure.
      if (et == 0) last_slice = atomicAdd(p.count + tile, 1u) == uint32_t(p.slices - 1);
      named_barrier(1, 128);
    }
    if (!CL && last_slice) {
      // Every slice's additions are in: dequantise this column tile and put
      // the accumulator and the counter back to zero.
      __threadfence();
      if (n < p.N) {
        const float ws = p.wscale[p.wscale_bcast ? 0 : n];
        float bs = 0.0f;
        if (HAS_BIAS) {
          if (p.bias_dtype == TG_DT_F32) bs = static_cast<const float*>(p.bias)[n];
          else if (p.bias_dtype == TG_DT_F16) bs = __half2float(static_cast<const __half*>(p.bias)[n]);
          else bs = __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
        }
        // Rows are finished 32 at a time: their sums are all loaded before any
        // is used, so the L2 latencies overlap instead of adding up.
        const size_t stride = size_t(p.N);
        int32_t* arow = p.acc + n;
        char* orow = static_cast<char*>(p.out) + size_t(n) * (OUT == 0 ? 4 : 2);
        const size_t ostride = stride * (OUT == 0 ? 4 : 2);
        constexpr int RB = MPAD < 32 ? MPAD : 32;
#pragma unroll 1
        for (int m0 = 0; m0 < MPAD; m0 += RB) {
          int32_t a[RB];
          {
            const int32_t* ap = arow;
#pragma unroll
            for (int j = 0; j < RB; ++j, ap += stride)
              if (m0 + j < p.M) a[j] = __ldcg(ap);
          }
          int32_t* zp = arow;
          char* o = orow;
#pragma unroll
          for (int j = 0; j < RB; ++j, zp += stride, o += ostride) {
            if (m0 + j < p.M) {
              __stcg(zp, 0);
              store_dequant<OUT, HAS_BIAS>(o, a[j], __ldg(p.xscale + m0 + j), ws, bs);
            }
          }
          arow += RB * stride;
          orow += RB * ostride;
        }
      }
      named_barrier(1, 128);
      if (et == 0) p.count[tile] = 0u;
    }
  }

  if (CL) {
    // Every CTA of the cluster reaches both barriers, also after a wait gave
    // up (its sums are then wrong, and the status word says so); the barriers
    // are warp-aligned, so each warp reconverges first.
    __syncwarp();
    cluster_sync();  // all partial tiles are in place
    if (warp >= 2) {
      const int nl = (warp & 3) * 32 + lane;
      const int n = n0 + nl;
      if (n < p.N) {
        const float ws = p.wscale[p.wscale_bcast ? 0 : n];
        float bs = 0.0f;
        if (HAS_BIAS) {
          if (p.bias_dtype == TG_DT_F32) bs = static_cast<const float*>(p.bias)[n];
          else if (p.bias_dtype == TG_DT_F16) bs = __half2float(static_cast<const __half*>(p.bias)[n]);
          else bs = __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
        }
        const int S = p.slices;  // 1..8
        // This lane's column of P in every CTA of the cluster (a CTA's window
        // is contiguous, so row m is at + m * 512 bytes).
        uint32_t peer[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          peer[q] = mapa_shared(smem_u32(smem) + uint32_t(nl) * 4u, uint32_t(q < S ? q : 0));
        char* o = static_cast<char*>(p.out) + size_t(n) * (OUT == 0 ? 4 : 2);
        const size_t ostride = size_t(p.N) * (OUT == 0 ? 4 : 2);
        // Rows rank, rank + S, ...: four rows' loads (up to 32) in flight at
        // once, so the distributed-shared-memory latencies overlap.
#pragma unroll 1
        for (int m = int(cluster_ctarank()); m < p.M; m += 4 * S) {
          int32_t part[4][8];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int mm = m + r * S;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              part[r][q] = (q < S && mm < p.M) ? ld_shared_cluster_s32(peer[q] + uint32_t(mm * BNW) * 4u) : 0;
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int mm = m + r * S;
            if (mm < p.M) {
              int32_t sum = 0;
#pragma unroll
              for (int q = 0; q < 8; ++q) sum += part[r][q];
              store_dequant<OUT, HAS_BIAS>(o + size_t(mm) * ostride, sum, __ldg(p.xscale + mm), ws, bs);
            }
          }
        }
      }
    }
    __syncwarp();
    cluster_sync();  // no CTA leaves while another still reads its shared memory
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // A wait gave up: let the loads still in flight (at most the last STAGES
  // issued, one per slot) land before the CTA exits.
  if (abort_flag && threadIdx.x == 0) {
    for (int i = max(0, issued - STAGES); i < issued; ++i)
      mbar_wait(&full_bar[i % STAGES], uint32_t(i / STAGES) & 1u, DEVERR_TMA_TIMEOUT);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace tg
