// INT8 GEMM with the int8_convrot dequantisation fused into the epilogue (sm_100a).
//
//   out[m,n] = ((float(sum_k xq[m,k]*wq[n,k]) * xscale[m]) * wscale[n]) + bias[n]
//
// the arithmetic of tilegen/quant/int8_ops.py:22-70 (torch._int_mm, then
// `.float()`, two `mul_`, `add_`, `copy_` to the output dtype), without the
// int32/fp32 temporaries: the int32 accumulators live in tensor memory and the
// fp32 epilogue runs on them in registers.
//
// Structure (persistent, one CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile [128 x 128 B] and B tile [BN(/2) x 128 B]
//               per k-block into a shared-memory ring (128-byte swizzle).
//   warp 1      allocates 512 TMEM columns; one lane issues tcgen05.mma kind::i8
//               (K=32 per instruction, four per k-block) into one of two int32
//               accumulators (TMEM columns 0 and 256), and commits each ring
//               slot back to the producer and each finished accumulator to the
//               epilogue.
//   warps 2-5   epilogue: tcgen05.ld 32 rows x one chunk of columns, int32 ->
//               fp32 (round to nearest), * xscale, * wscale, + bias, convert,
//               then a swizzled shared-memory chunk stored by a TMA bulk tensor
//               store (two staging chunks per warp where shared memory allows,
//               so a chunk's conversion overlaps the previous chunk's store).
// PAIR = false: each CTA computes a 128 x BN tile (cta_group::1, M=128).
// PAIR = true: the two CTAs of a cluster compute one 256 x BN tile with the
//   pair MMA (cta_group::2, M=256): each CTA loads its 128 rows of A and half
//   (BN/2 rows) of B, so per SM the operand traffic per MMA is a third lower.
//   Both CTAs' loads complete on the even CTA's ring barriers; its MMA thread
//   issues for the pair and its commits arrive on both CTAs' barriers; both
//   epilogues release an accumulator by arriving on the even CTA's barrier.
// Tiles are walked M-fastest within groups of 16 m-tiles (tile_coords), so the
// CTAs in flight share weight columns in L2 and A stays in L2 across a group.
// Every mbarrier wait is bounded (see common.cuh); a role that gives up stops
// the others in its CTA, and the peer CTA's waits then expire as well.
#pragma once

#include "common.cuh"

namespace tg {

namespace gemm {
constexpr int BM = 128;               // rows of xq per CTA (UMMA M per CTA)
constexpr int BN_MAX = 256;           // widest tile (rows of wq per tile, UMMA N)
constexpr int BK = 128;               // bytes (= int8 elements) of K per k-block
constexpr int UK = 32;                // K per tcgen05.mma kind::i8
constexpr int A_BYTES = BM * BK;      // 16 KB
constexpr int OUT_BYTES = 32 * 128;   // one 32-row x 128-byte epilogue chunk per warp
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;        // two accumulators, at columns 0 and 256
constexpr uint32_t SMEM_LIMIT = 232448;

// Rows of B each CTA holds; 128-byte K sub-blocks per ring slot (pair tiles
// take two, so the MMA thread waits once per 8 MMAs: a barrier wait costs the
// issuing thread a few hundred cycles, more than 4 MMAs of a 128-row tile
// take); bytes of one slot; ring depth; dynamic shared memory.
__host__ __device__ constexpr int b_rows(int bn, bool pair) { return pair ? bn / 2 : bn; }
__host__ __device__ constexpr int ksub(bool pair) { return pair ? 2 : 1; }
__host__ __device__ constexpr uint32_t stage_bytes(int bn, bool pair) {
  return uint32_t(ksub(pair) * (A_BYTES + b_rows(bn, pair) * BK));
}
__host__ __device__ constexpr int stages_with(int bn, bool pair, int nbuf) {
  return int((SMEM_LIMIT - 4 * nbuf * OUT_BYTES - 1024 - 4096) / stage_bytes(bn, pair)) > 8
             ? 8
             : int((SMEM_LIMIT - 4 * nbuf * OUT_BYTES - 1024 - 4096) / stage_bytes(bn, pair));
}
// Staging chunks per epilogue warp: two (one is converted while the TMA store
// of the other reads it) when the second costs the operand ring no slot, else
// one.  Two for the 160- to 224-wide pair tiles, one for 256 and 128.
__host__ __device__ constexpr int out_bufs(int bn, bool pair) {
  return stages_with(bn, pair, 2) >= stages_with(bn, pair, 1) ? 2 : 1;
}
__host__ __device__ constexpr int stages(int bn, bool pair) { return stages_with(bn, pair, out_bufs(bn, pair)); }
__host__ __device__ constexpr uint32_t smem_bytes(int bn, bool pair) {
  return uint32_t(stages(bn, pair)) * stage_bytes(bn, pair) + uint32_t(4 * out_bufs(bn, pair)) * OUT_BYTES + 1024;
}

// tcgen05 instruction descriptor: D=S32 (bits 4-5 = 2), A=B=S8 (bits 7-9 and
// 10-12 = 1), both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
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
  int m_tiles, n_tiles, k_blocks;  // m_tiles: 128-row (single) or 256-row (pair) tiles;
                                   // k_blocks: ring slots of ksub(pair) * 128 bytes of K
};

// m-tiles per group of the tile order: 16 (4096 rows of A in pair tiles) keeps
// a group's A in L2 while its column tiles stream past.
constexpr int kTileGroupM = 16;

// Tile t -> (m-tile, n-tile).  Groups of kTileGroupM m-tiles, one after the
// other; inside a group tiles go M-fastest, so the CTAs in flight share weight
// columns in L2 and A is read from HBM about once (a plain M-fastest order
// over a large M would read all of A again for every column tile).
__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& mt, int& nt) {
  const int per_group = kTileGroupM * p.n_tiles;
  const int group = t / per_group;
  const int first = group * kTileGroupM;
  const int size = min(kTileGroupM, p.m_tiles - first);
  const int r = t - group * per_group;
  mt = first + r % size;
  nt = r / size;
}

// BN: tile width (a multiple of 32, at most 256); OUT: 0 fp32, 1 fp16, 2 bf16
// (tg_dtype codes); PAIR: see above (launched with clusters of 2 CTAs).
template <int BN, int OUT, bool HAS_BIAS, bool PAIR>
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
  constexpr int S = stages(BN, PAIR);
  constexpr int NBUF = out_bufs(BN, PAIR);
  constexpr int BROWS = b_rows(BN, PAIR);
  constexpr int KS = ksub(PAIR);
  constexpr uint32_t B_BYTES = uint32_t(BROWS) * BK;       // one 128-byte K sub-block of B
  constexpr uint32_t A_SLOT = uint32_t(KS) * A_BYTES;       // ring slot of A
  constexpr uint32_t B_SLOT = uint32_t(KS) * B_BYTES;       // ring slot of B
  constexpr int TILE_M = PAIR ? 2 * BM : BM;
  constexpr uint32_t IDESC = idesc(TILE_M, BN);
  constexpr uint32_t TX_BYTES = (PAIR ? 2u : 1u) * (A_SLOT + B_SLOT);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * A_SLOT;
  uint8_t* sOut = sB + S * B_SLOT;

  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ __align__(16) float col_ws[BN_MAX];
  __shared__ __align__(16) float col_bias[BN_MAX];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);   // tile-processing unit
  const int units = PAIR ? int(gridDim.x >> 1) : int(gridDim.x);
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
    prefetch_tmap(&tma_out);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], PAIR ? 8 : 4);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(&tmem_base_sh, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&tmem_base_sh, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (PAIR) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  // Everything above overlaps the tail of the kernel that produced xq/xscale
  // (when launched as its programmatic dependent); nothing below may read them
  // before it has completed.
  pdl_wait();

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
      for (int t = unit; t < num_tiles; t += units) {
        int mt, nt;
        tile_coords(t, p, mt, nt);
        const int m0 = mt * TILE_M + int(rank) * BM;
        const int n0 = nt * BN + int(rank) * BROWS;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait(&empty_bar[stage], phase ^ 1u, DEVERR_PIPE_TIMEOUT)) goto done;
          if (PAIR) {
            // Both CTAs' copies land on the even CTA's barrier, which expects
            // the bytes of both.
            const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], TX_BYTES);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
              const int kx = (kb * KS + ks) * BK;
              tma_load_2d_pair(sA + stage * A_SLOT + ks * A_BYTES, &tma_a, fb, kx, m0);
              tma_load_2d_pair(sB + stage * B_SLOT + ks * B_BYTES, &tma_b, fb, kx, n0);
            }
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], TX_BYTES);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
              const int kx = (kb * KS + ks) * BK;
              tma_load_2d(sA + stage * A_SLOT + ks * A_BYTES, &tma_a, &full_bar[stage], kx, m0);
              tma_load_2d(sB + stage * B_SLOT + ks * B_BYTES, &tma_b, &full_bar[stage], kx, n0);
            }
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = unit; t < num_tiles; t += units, ++local) {
        const int ab = local & 1;
        const uint32_t acc_phase = uint32_t(local >> 1) & 1u;
        if (!wait(&tempty_bar[ab], acc_phase ^ 1u, DEVERR_PIPE_TIMEOUT)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(ab * BN_MAX);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait(&full_bar[stage], phase, DEVERR_TMA_TIMEOUT)) goto done;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_SLOT);
          const uint32_t b_addr = smem_u32(sB + stage * B_SLOT);
#pragma unroll
          for (int k = 0; k < KS * (BK / UK); ++k) {
            const int ks = k / (BK / UK), kk = k % (BK / UK);
            const uint64_t ad = kmajor_sw128_desc(a_addr + ks * A_BYTES + kk * UK);
            const uint64_t bd = kmajor_sw128_desc(b_addr + ks * B_BYTES + kk * UK);
            const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
            if (PAIR) mma_i8_pair(d_tmem, ad, bd, IDESC, acc);
            else mma_i8(d_tmem, ad, bd, IDESC, acc);
          }
          // The slot is free once these MMAs have read it (in both CTAs).
          if (PAIR) mma_commit_pair(&empty_bar[stage], 0x3); else mma_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        // Accumulator complete (both CTAs' halves).
        if (PAIR) mma_commit_pair(&tfull_bar[ab], 0x3); else mma_commit(&tfull_bar[ab]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 64;      // 0..127
    const int quarter = warp & 3;         // TMEM lanes [32*quarter, +32)
    uint8_t* const sbufs = sOut + (warp - 2) * NBUF * OUT_BYTES;
    int chunk_seq = 0;  // chunks this warp has staged; every chunk commits one bulk group
    const uint32_t tempty_leader0 = PAIR ? mapa_shared(smem_u32(&tempty_bar[0]), 0) : 0u;
    const uint32_t tempty_leader1 = PAIR ? mapa_shared(smem_u32(&tempty_bar[1]), 0) : 0u;
    int local = 0;
    for (int t = unit; t < num_tiles; t += units, ++local) {
      int mt, nt;
      tile_coords(t, p, mt, nt);
      const int m0 = mt * TILE_M + int(rank) * BM;
      const int n0 = nt * BN;
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

      // One chunk of columns: tcgen05.ld of 32 lanes x CH columns, dequantise,
      // stage, TMA store.  The next chunk's tensor-memory load is issued before
      // this chunk is converted, so its latency overlaps the conversion.
      auto load_chunk = [&](uint32_t (&acc)[CH], int ch) {
#pragma unroll
        for (int h = 0; h < CH / 32; ++h)
          tmem_ld_32x32b_x32(t_row + uint32_t(ch * CH + h * 32), *reinterpret_cast<uint32_t(*)[32]>(&acc[h * 32]));
      };
      auto store_chunk = [&](const uint32_t (&acc)[CH], int ch) {
        // The TMA store that last used this staging chunk (NBUF chunks ago)
        // must have finished reading it; later stores may still be in flight.
        uint8_t* const sbuf = sbufs + (chunk_seq % NBUF) * OUT_BYTES;
        ++chunk_seq;
        if (lane == 0) bulk_wait_read<NBUF - 1>();
        __syncwarp();

        const float* cws = col_ws + ch * CH;
        const float* cbs = col_bias + ch * CH;
        uint8_t* srow = sbuf + lane * CH_BYTES;
#pragma unroll
        for (int c16 = 0; c16 < CH_BYTES / 16; ++c16) {  // 16 output bytes per step
          uint32_t pk[4];
          constexpr int PER = 16 / ESZ;                  // values per 16 bytes
#pragma unroll
          for (int e = 0; e < PER; e += 4) {
            const int j = c16 * PER + e;
            const float4 w4 = *reinterpret_cast<const float4*>(cws + j);
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (HAS_BIAS) b4 = *reinterpret_cast<const float4*>(cbs + j);
            float r[4];
            if (HAS_BIAS) {
              // Scalar: a paired multiply followed by a paired add may be
              // contracted into one fma, which would round once.
              const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
              const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                float v = __int2float_rn(static_cast<int>(acc[j + u]));
                v = __fmul_rn(v, xs);
                v = __fmul_rn(v, wv[u]);
                r[u] = __fadd_rn(v, bv[u]);
              }
            } else {
              // Two columns per paired multiply: each lane one IEEE rounding,
              // as the scalar (float(acc) * xs) * ws.
              const float2 xs2 = make_float2(xs, xs);
              float2 r01 = make_float2(__int2float_rn(static_cast<int>(acc[j])),
                                       __int2float_rn(static_cast<int>(acc[j + 1])));
              float2 r23 = make_float2(__int2float_rn(static_cast<int>(acc[j + 2])),
                                       __int2float_rn(static_cast<int>(acc[j + 3])));
              r01 = mul2(mul2(r01, xs2), make_float2(w4.x, w4.y));
              r23 = mul2(mul2(r23, xs2), make_float2(w4.z, w4.w));
              r[0] = r01.x;
              r[1] = r01.y;
              r[2] = r23.x;
              r[3] = r23.y;
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
        // A box that starts past the last row/column would store nothing; skip
        // it, but still commit a (then empty) group so that the count of
        // groups behind each staging chunk stays one per chunk.
        if (lane == 0) {
          if (m0 + quarter * 32 < p.M && n0 + ch * CH < p.N)
            tma_store_2d(&tma_out, sbuf, n0 + ch * CH, m0 + quarter * 32);
          bulk_commit();
        }
      };
      uint32_t acc_a[CH], acc_b[CH];
      load_chunk(acc_a, 0);
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        uint32_t(&cur)[CH] = (ch & 1) ? acc_b : acc_a;
        uint32_t(&nxt)[CH] = (ch & 1) ? acc_a : acc_b;
        tmem_wait_ld();
        reg_after_wait(cur);
        if (ch + 1 < NCH) {
          load_chunk(nxt, ch + 1);
        } else {
          // This warp is done reading the accumulator: hand it back to the MMA.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (PAIR) mbar_arrive_cluster(ab ? tempty_leader1 : tempty_leader0);
            else mbar_arrive(&tempty_bar[ab]);
          }
        }
        store_chunk(cur, ch);
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

done:
  __syncwarp();
  tc_fence_before();
  // Neither CTA of a pair may leave while the other can still touch its
  // shared memory or tensor memory.
  if (PAIR) cluster_sync(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace tg
