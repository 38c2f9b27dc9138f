// INT8 GEMM with the int8_convrot dequantisation fused into the epilogue (sm_100a).
//
//   out[m,n] = ((float(sum_k xq[m,k]*wq[n,k]) * xscale[m]) * wscale[n]) + bias[n]
//
// the arithmetic of tilegen/quant/int8_ops.py:22-70 (torch._int_mm, then
// `.float()`, two `mul_`, `add_`, `copy_` to the output dtype), without the
// int32/fp32 temporaries: the int32 accumulators live in tensor memory and the
// fp32 epilogue runs on them in registers.
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile [128 x 128 B] and B tile [256 x 128 B] per
//               k-block into a 4-deep shared-memory ring (128-byte swizzle).
//   warp 1      allocates 512 TMEM columns; one lane issues tcgen05.mma
//               kind::i8 (M=128, N=256, K=32; four per k-block) into one of two
//               256-column int32 accumulators, and commits each ring slot back
//               to the producer and each finished accumulator to the epilogue.
//   warps 2-5   epilogue: tcgen05.ld 32 rows x 64 columns at a time, int32 ->
//               fp32 (round to nearest), * xscale, * wscale, + bias, convert, and
//               a swizzled shared-memory tile stored with a TMA bulk tensor store.
// Tiles are walked M-fastest so the CTAs in flight share the same weight
// columns in L2.  Two accumulators let the epilogue of tile i overlap the MMAs
// of tile i+1.  Every mbarrier wait is bounded (see common.cuh).
#pragma once

#include "common.cuh"

namespace tg {

namespace gemm {
constexpr int BM = 128;               // rows of xq per tile (UMMA M)
constexpr int BN_MAX = 256;           // widest tile (rows of wq per tile, UMMA N)
constexpr int BK = 128;               // bytes (= int8 elements) of K per k-block
constexpr int UK = 32;                // K per tcgen05.mma kind::i8
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;      // 16 KB
constexpr int OUT_BYTES = 32 * 128;   // one 32-row x 128-byte epilogue chunk per warp
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;        // two accumulators, at columns 0 and 256

template <int BN>
__host__ __device__ constexpr uint32_t smem_bytes() {
  return STAGES * (A_BYTES + BN * BK) + 4 * OUT_BYTES + 1024;
}

// tcgen05 instruction descriptor: D=S32 (bits 4-5 = 2), A=B=S8 (bits 7-9 and
// 10-12 = 1), both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
template <int BN>
__host__ __device__ constexpr uint32_t idesc() {
  return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major operand tile stored as rows
// of 128 bytes in the 128-byte swizzle: start address >> 4, leading byte
// offset 16 B (unused by this layout), stride byte offset 1024 B between
// 8-row swizzle atoms, descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3fffu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
}  // namespace gemm

struct GemmParams {
  const float* xscale;
  const float* wscale;
  const void* bias;
  int bias_dtype;  // tg_dtype
  int wscale_bcast;
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
};

// BN: tile width (a multiple of 32, at most 256); OUT: 0 fp32, 1 fp16, 2 bf16
// (tg_dtype codes).
template <int BN, int OUT, bool HAS_BIAS>
__global__ void __launch_bounds__(gemm::THREADS, 1)
    gemm_i8_dequant_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                           const __grid_constant__ CUtensorMap tma_out, const GemmParams p) {
  using namespace gemm;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= BN_MAX, "tile width");
  constexpr int ESZ = OUT == 0 ? 4 : 2;
  // Epilogue chunk: 128-byte rows (128-byte swizzle) when the tile width
  // allows, else 64-byte rows (64-byte swizzle).
  constexpr int CH_BYTES = (BN * ESZ) % 128 == 0 ? 128 : 64;
  constexpr int CH = CH_BYTES / ESZ;   // output columns per epilogue chunk
  constexpr int NCH = BN / CH;         // chunks per tile
  constexpr int B_BYTES = BN * BK;
  constexpr uint32_t IDESC = idesc<BN>();

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * B_BYTES;

  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ __align__(16) float col_ws[BN_MAX];
  __shared__ __align__(16) float col_bias[BN_MAX];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
    prefetch_tmap(&tma_out);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  // Bounded wait that also gives up as soon as another role has given up.
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
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int m0 = (t % p.m_tiles) * BM;
        const int n0 = (t / p.m_tiles) * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait(&empty_bar[stage], phase ^ 1u, DEVERR_PIPE_TIMEOUT)) goto done;
          mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tma_a, &full_bar[stage], kb * BK, m0);
          tma_load_2d(sB + stage * B_BYTES, &tma_b, &full_bar[stage], kb * BK, n0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
        const int ab = local & 1;
        const uint32_t acc_phase = uint32_t(local >> 1) & 1u;
        if (!wait(&tempty_bar[ab], acc_phase ^ 1u, DEVERR_PIPE_TIMEOUT)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(ab * BN_MAX);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait(&full_bar[stage], phase, DEVERR_TMA_TIMEOUT)) goto done;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UK; ++k) {
            mma_i8(d_tmem, kmajor_sw128_desc(a_addr + k * UK), kmajor_sw128_desc(b_addr + k * UK), IDESC,
                   (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty_bar[stage]);  // slot is free once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        mma_commit(&tfull_bar[ab]);  // accumulator complete
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 64;      // 0..127
    const int quarter = warp & 3;         // TMEM lanes [32*quarter, +32)
    uint8_t* sbuf = sOut + (warp - 2) * OUT_BYTES;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int m0 = (t % p.m_tiles) * BM;
      const int n0 = (t / p.m_tiles) * BN;
      const int ab = local & 1;
      // Column parameters of this tile (shared by the four epilogue warps).
      named_barrier(1, 128);
      for (int c = et; c < BN; c += 128) {
        const int n = n0 + c;
        float ws = 0.0f, bs = 0.0f;
        if (n < p.N) {
          ws = p.wscale[p.wscale_bcast ? 0 : n];
          if (HAS_BIAS) {
            if (p.bias_dtype == TG_DT_F32) bs = static_cast<const float*>(p.bias)[n];
            else if (p.bias_dtype == TG_DT_F16) bs = __half2float(static_cast<const __half*>(p.bias)[n]);
            else bs = __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
          }
        }
        col_ws[c] = ws;
        col_bias[c] = bs;
      }
      named_barrier(1, 128);

      if (!wait(&tfull_bar[ab], uint32_t(local >> 1) & 1u, DEVERR_MMA_TIMEOUT)) break;
      tc_fence_after();

      const int row = m0 + quarter * 32 + lane;
      const float xs = row < p.M ? p.xscale[row] : 0.0f;
      const uint32_t t_row = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(ab * BN_MAX);

#pragma unroll 1
      for (int ch = 0; ch < NCH; ++ch) {
        uint32_t acc[CH];
#pragma unroll
        for (int h = 0; h < CH / 32; ++h)
          tmem_ld_32x32b_x32(t_row + uint32_t(ch * CH + h * 32), *reinterpret_cast<uint32_t(*)[32]>(&acc[h * 32]));
        tmem_wait_ld();
        if (ch == NCH - 1) {
          // This warp is done reading the accumulator: hand it back to the MMA.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[ab]);
        }
        // The previous chunk's TMA store must have finished reading sbuf.
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();

        const float* cws = col_ws + ch * CH;
        const float* cbs = col_bias + ch * CH;
        uint8_t* srow = sbuf + lane * CH_BYTES;
#pragma unroll
        for (int c16 = 0; c16 < CH_BYTES / 16; ++c16) {  // 16 output bytes per step
          uint32_t pk[4];
          constexpr int PER = 16 / ESZ;       // values per 16 bytes
#pragma unroll
          for (int e = 0; e < PER; e += 4) {
            const int j = c16 * PER + e;
            const float4 w4 = *reinterpret_cast<const float4*>(cws + j);
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (HAS_BIAS) b4 = *reinterpret_cast<const float4*>(cbs + j);
            const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
            const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
            float r[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              float v = __int2float_rn(static_cast<int>(acc[j + u]));
              v = __fmul_rn(v, xs);
              v = __fmul_rn(v, wv[u]);
              if (HAS_BIAS) v = __fadd_rn(v, bv[u]);
              r[u] = v;
            }
            if (OUT == 0) {
#pragma unroll
              for (int u = 0; u < 4; ++u) pk[e + u] = __float_as_uint(r[u]);
            } else if (OUT == 1) {
              __half2 h0 = __floats2half2_rn(r[0], r[1]);
              __half2 h1 = __floats2half2_rn(r[2], r[3]);
              pk[e / 2] = *reinterpret_cast<uint32_t*>(&h0);
              pk[e / 2 + 1] = *reinterpret_cast<uint32_t*>(&h1);
            } else {
              __nv_bfloat162 h0 = __floats2bfloat162_rn(r[0], r[1]);
              __nv_bfloat162 h1 = __floats2bfloat162_rn(r[2], r[3]);
              pk[e / 2] = *reinterpret_cast<uint32_t*>(&h0);
              pk[e / 2 + 1] = *reinterpret_cast<uint32_t*>(&h1);
            }
          }
          // 128-byte swizzle: chunk ^= row & 7; 64-byte swizzle: chunk ^= (row >> 1) & 3.
          const uint32_t pc = CH_BYTES == 128 ? (uint32_t(c16) ^ uint32_t(lane & 7))
                                              : (uint32_t(c16) ^ uint32_t((lane >> 1) & 3));
          *reinterpret_cast<uint4*>(srow + (pc << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        // A box that starts past the last row/column would store nothing; skip it.
        if (lane == 0 && m0 + quarter * 32 < p.M && n0 + ch * CH < p.N) {
          tma_store_2d(&tma_out, sbuf, n0 + ch * CH, m0 + quarter * 32);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

done:
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace tg
