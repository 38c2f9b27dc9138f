// Fused group-Hadamard rotation + row-wise int8 quantisation (sm_100a).
//
// Algorithm (the reference kernel `fht_quant`, tilegen/kernels/int8_convrot.py:47-104):
// per group of G = 4^NST elements, NST radix-4 butterfly stages on the H4 of
// tilegen/kernels/hadamard.py:15, stage s at stride 4^s; then the row absmax,
// the scale absmax/(127*sqrt(G)) clamped at 1e-30, and codes
// rint(v / (sqrt(G)*scale)).  Two fp32 evaluation orders (EXACT):
//  * EXACT: every output summed left to right as at int8_convrot.py:74-77, the
//    product rounded and clamped: the same operations in the same order, so
//    codes and scales are bit-identical to that kernel (and to the C oracle's
//    oracle_rotate_quant);
//  * short (the default): each output S - 2*a_i in one fma (bfly4x2_short) and
//    the code rint(v*inv) as one fma for finite rows: fewer roundings, codes
//    within one of the reference order's at rounding ties (bit-identical to the
//    oracle's oracle_rotate_quant_short).
//
// B200 layout:
//  * A persistent CTA owns R rows at a time ("a batch").  One thread owns one
//    64-element chunk of a row (its 128-byte "line"), so a row is K/64 threads
//    and a batch is R*K/64 threads; R is picked so the batch fills whole warps.
//  * Batches stream HBM -> shared memory with 2-D TMA copies (128-byte swizzle)
//    into a ring of `stages` buffers completed on mbarriers, so several batches
//    are in flight per SM while the current one is rotated.
//  * Stages 0..2 (index bits 0..5) run in registers on the thread's own 64
//    values.  For G=256 stage 3 needs the four chunks of a group: the four
//    threads swap 16-value blocks through the warp's own (already consumed)
//    slice of the stage buffer, so that afterwards each holds one 16-wide
//    column block for all four inputs of the last butterfly, in input order.
//  * Row absmax: warp shuffles over the row's lanes, then one shared-memory
//    atomicMax per segment and a CTA barrier.  The rotated values never leave
//    registers; the codes are packed 16 per 128-bit store straight to HBM.
//
// Two prologue/branch options of the production wrapper
// (tilegen/comfyui/backend.py:166-244) run inside the same pass:
//  * ACT: an elementwise input activation applied to x before anything else
//    (backend.py:201-204), evaluated in fp32 and rounded back to x's dtype as
//    the separate elementwise op it replaces would store it;
//  * NST == 0: no rotation -- the row-wise int8 branch of backend.py:230-232,
//    with that branch's torch arithmetic (scale = absmax * fp32(1/127) clamped
//    at 1e-30, codes = int8(clamp(round(dtype(x / dtype(scale))), -128, 127)),
//    NaN propagating through absmax as torch's amax does).
#pragma once

#include "common.cuh"

namespace tg {

struct RotQuantParams {
  int8_t* q;
  float* scale;
  int64_t M;
  int K;
  int cpr;               // 64-element chunks per row = K / 64
  int rows_per_batch;    // R
  int active;            // threads that own a chunk = R * cpr
  int box_lines;         // 128-byte lines per TMA box
  int boxes;             // TMA boxes per batch
  int64_t nbatches;      // ceil(M / R)
  int stages;            // shared-memory ring depth
  uint32_t stage_bytes;  // bytes per ring slot = blockDim.x * 128 (a multiple of 1024)
  int seg;               // lanes per absmax shuffle segment = gcd(cpr, 32)
  // kActLnMod only: modulation vectors [ceil(M / mod_rows), K] of x's dtype
  // (rows r use vector r / mod_rows) and the LayerNorm epsilon.
  const void* mod_scale;
  const void* mod_shift;
  int64_t mod_rows;
  float ln_eps;
  float ln_inv_k;  // RN(1 / K): the mean and the variance are sums times it
};

// Words of shared memory the LayerNorm prologue needs beyond the ring, the
// barriers and the row maxima: per-line partial sums of x and of (x - mean)^2
// ([R][lines]) and their 16 column sums ([R][16]), for a CTA of `threads`
// threads (lines <= threads / R), plus 4 words of slack to align them to 16 bytes.
__host__ __device__ constexpr int ln_words(int threads, int R) { return 2 * threads + 2 * 16 * R + 4; }

// Packed round-to-nearest add and multiply of two x-dtype pairs held as the
// bits of 32-bit words.
template <bool BF16>
__device__ __forceinline__ uint32_t hadd2_dt(uint32_t a, uint32_t b) {
  uint32_t r;
  if (BF16) asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <bool BF16>
__device__ __forceinline__ uint32_t hmul2_dt(uint32_t a, uint32_t b) {
  uint32_t r;
  if (BF16) asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  // Opaque to the compiler: the product is rounded on its own, never
  // contracted with the add that follows into one fma.
  asm volatile("" : "+r"(r));
  return r;
}

// Sum of one row's per-line partials in a fixed order: column c < 16 of the
// row adds lines c, c + 16, c + 32, ... (ascending) into col[c] (columns past
// the row's lines stay 0: zeroed once at kernel start), then every thread adds
// the 16 columns as a pairwise tree, ((c0 + c1) + (c2 + c3)) + ... .  Two CTA
// barriers; every thread of the CTA must call it.  `part` [R][lines], `col`
// [R][16] (16-byte aligned).
__device__ __forceinline__ float row_total(float* part, float* col, float mine, bool active, int row_local,
                                           int chunk, int cpr) {
  if (active) part[row_local * cpr + chunk] = mine;
  __syncthreads();
  if (active && chunk < 16) {
    // Loads four lines ahead of the (sequential) adds, so that their shared-
    // memory latencies overlap while the other threads wait at the barrier.
    const float* pr = part + row_local * cpr;
    float t = pr[chunk];
    int c = chunk + 16;
    for (; c + 48 < cpr; c += 64) {
      const float a = pr[c], b = pr[c + 16], d = pr[c + 32], e = pr[c + 48];
      t = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(t, a), b), d), e);
    }
    for (; c < cpr; c += 16) t = __fadd_rn(t, pr[c]);
    col[row_local * 16 + chunk] = t;
  }
  __syncthreads();
  const float4* c4 = reinterpret_cast<const float4*>(col + row_local * 16);
  float4 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = active ? c4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  float q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = __fadd_rn(__fadd_rn(v[i].x, v[i].y), __fadd_rn(v[i].z, v[i].w));
  return __fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3]));
}

// One radix-4 butterfly, each output evaluated exactly as
//   y0 = a0 + a1 + a2 - a3, y1 = a0 + a1 - a2 + a3,
//   y2 = a0 - a1 + a2 + a3, y3 = -a0 + a1 + a2 + a3   (left to right),
// with the shared partial sums factored out: (-a0 + a1) == -(a0 - a1) and
// (-d) + a2 == a2 - d hold exactly in IEEE arithmetic.
__device__ __forceinline__ void bfly4(float& a0, float& a1, float& a2, float& a3) {
  const float s = __fadd_rn(a0, a1);
  const float d = __fsub_rn(a0, a1);
  const float y0 = __fsub_rn(__fadd_rn(s, a2), a3);
  const float y1 = __fadd_rn(__fsub_rn(s, a2), a3);
  const float y2 = __fadd_rn(__fadd_rn(d, a2), a3);
  const float y3 = __fadd_rn(__fsub_rn(a2, d), a3);
  a0 = y0;
  a1 = y1;
  a2 = y2;
  a3 = y3;
}

// bfly4 on two independent butterflies at once (lanes .x and .y).
__device__ __forceinline__ void bfly4x2(float2& a0, float2& a1, float2& a2, float2& a3) {
  const float2 s = add2(a0, a1);
  const float2 d = sub2(a0, a1);
  const float2 y0 = sub2(add2(s, a2), a3);
  const float2 y1 = add2(sub2(s, a2), a3);
  const float2 y2 = add2(add2(d, a2), a3);
  const float2 y3 = add2(sub2(a2, d), a3);
  a0 = y0;
  a1 = y1;
  a2 = y2;
  a3 = y3;
}

// max(m, |a|, |b|) in one three-input max; NaN operands are ignored as by fmaxf.
__device__ __forceinline__ float absmax3(float m, float a, float b) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return r;
}

// The same with NaN propagating: NaN when any operand is NaN.
__device__ __forceinline__ float absmax3_nan(float m, float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return r;
}

// ---- the short butterfly (default order) -------------------------------------
// The same H4 product with fewer roundings per output:
//   S = (a0 + a2) + (a1 + a3),   y_{3-i} = S - 2 a_i   (one fma each),
// because every row of the H4 is all ones but one -1, at column 3 - i for row i.
// Written in place, position i of the digit ends up holding output 3 - i, so
// after all stages of a group position P holds output G - 1 - P (each base-4
// digit reversed); the stores undo that.  3 adds and 4 fmas per 4 outputs
// against the 10 adds of the reference order; the results differ from that
// order by a few fp32 ulps, so codes can differ by one at rounding ties.
__device__ __forceinline__ void bfly4x2_short(float2& a0, float2& a1, float2& a2, float2& a3) {
  const float2 s = add2(add2(a0, a2), add2(a1, a3));
  const float2 m2 = make_float2(-2.0f, -2.0f);
  a0 = fma2(a0, m2, s);
  a1 = fma2(a1, m2, s);
  a2 = fma2(a2, m2, s);
  a3 = fma2(a3, m2, s);
}

// One butterfly whose inputs are two pairs p0 = (a0, a1), p1 = (a2, a3):
// t = (a0 + a2, a1 + a3) paired, S formed in both lanes (t.x + t.y and
// t.y + t.x are the same IEEE sum), then the two fmas paired.
__device__ __forceinline__ void bfly4_short(float2& p0, float2& p1) {
  const float2 t = add2(p0, p1);
  const float2 s = make_float2(__fadd_rn(t.x, t.y), __fadd_rn(t.y, t.x));
  const float2 m2 = make_float2(-2.0f, -2.0f);
  p0 = fma2(p0, m2, s);
  p1 = fma2(p1, m2, s);
}

__device__ __forceinline__ void stage0_64_short(float2 (&vp)[32]) {
#pragma unroll
  for (int h = 0; h < 16; ++h) bfly4_short(vp[2 * h], vp[2 * h + 1]);
}

__device__ __forceinline__ void stage1_64_short(float2 (&vp)[32]) {
#pragma unroll
  for (int h = 0; h < 4; ++h)
#pragma unroll
    for (int u = 0; u < 2; ++u)
      bfly4x2_short(vp[8 * h + u], vp[8 * h + 2 + u], vp[8 * h + 4 + u], vp[8 * h + 6 + u]);
}

__device__ __forceinline__ void stage2_64_short(float2 (&vp)[32]) {
#pragma unroll
  for (int l = 0; l < 8; ++l) bfly4x2_short(vp[l], vp[l + 8], vp[l + 16], vp[l + 24]);
}

// The thread's 64 values are held as 32 pairs vp[k] = (v[2k], v[2k+1]).
// Stage 0 (stride 1) pairs two inputs of one butterfly, so it runs scalar;
// stages 1 and 2 (strides 4 and 16) pair the butterflies at positions p and
// p+1, which are independent and identical, so they run on f32x2.
__device__ __forceinline__ void stage0_64(float2 (&vp)[32]) {
#pragma unroll
  for (int h = 0; h < 16; ++h) bfly4(vp[2 * h].x, vp[2 * h].y, vp[2 * h + 1].x, vp[2 * h + 1].y);
}

__device__ __forceinline__ void stage1_64(float2 (&vp)[32]) {
#pragma unroll
  for (int h = 0; h < 4; ++h)
#pragma unroll
    for (int u = 0; u < 2; ++u) bfly4x2(vp[8 * h + u], vp[8 * h + 2 + u], vp[8 * h + 4 + u], vp[8 * h + 6 + u]);
}

__device__ __forceinline__ void stage2_64(float2 (&vp)[32]) {
#pragma unroll
  for (int l = 0; l < 8; ++l) bfly4x2(vp[l], vp[l + 8], vp[l + 16], vp[l + 24]);
}

// Input operations applied to x before the rotation: the activations (the
// names of backend.py's `input_act`), and kActLnMod, the DiT block's
// LayerNorm (no affine) followed by its modulation, y = LN(x) * (1 + scale) + shift.
enum : int { kActNone = 0, kActGeluTanh = 1, kActGelu = 2, kActLnMod = 3 };

// The activation in fp32 on a pair, written as torch's CUDA GELU kernels
// evaluate it in their fp32 op-math -- the same operations in the same order
// (x_cube = (x*x)*x; inner = kBeta * fma(kKappa, x_cube, x), the contraction
// the compiler makes of `x + kKappa * x_cube`; the same tanhf/erff calls, each
// followed by the scalar `1 + ...`) -- with the multiplies of the two lanes
// paired:
//   gelu_tanh(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
//   gelu(x)      = x 0.5 (1 + erf(x / sqrt(2)))
template <int ACT>
__device__ __forceinline__ float2 act2_f32(float2 x) {
  if (ACT == kActGeluTanh) {
    constexpr float kBeta = float(1.41421356237309504880 * 1.12837916709551257390 * 0.5);
    constexpr float kKappa = 0.044715f;
    const float2 x_cube = mul2(mul2(x, x), x);
    const float2 inner = mul2(make_float2(kBeta, kBeta), fma2(make_float2(kKappa, kKappa), x_cube, x));
    const float2 one_t = make_float2(1.0f + tanhf(inner.x), 1.0f + tanhf(inner.y));
    return mul2(mul2(make_float2(0.5f, 0.5f), x), one_t);
  } else if (ACT == kActGelu) {
    constexpr float kAlpha = float(0.70710678118654752440);
    const float2 xa = mul2(x, make_float2(kAlpha, kAlpha));
    const float2 one_e = make_float2(1.0f + erff(xa.x), 1.0f + erff(xa.y));
    return mul2(mul2(x, make_float2(0.5f, 0.5f)), one_e);
  }
  return x;
}

// fp32 -> x's dtype -> fp32 (round to nearest even), as a store to an
// fp16/bf16 tensor and the next op's load do.
template <bool BF16>
__device__ __forceinline__ float round_to_dtype(float v) {
  return BF16 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}

// The same for a pair, as one packed conversion (cvt.rn.{f16,bf16}x2.f32).
template <bool BF16>
__device__ __forceinline__ uint32_t pack2_dtype(float2 v) {
  if (BF16) {
    const __nv_bfloat162 h = __float22bfloat162_rn(v);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __half2 h = __float22half2_rn(v);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2_dtype(uint32_t u) {
  if (BF16) return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}

template <bool BF16, int ACT>
__device__ __forceinline__ void unpack8(const uint4 w, float2* f) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[i] = unpack2_dtype<BF16>(u[i]);
    if (ACT == kActGeluTanh || ACT == kActGelu) f[i] = unpack2_dtype<BF16>(pack2_dtype<BF16>(act2_f32<ACT>(f[i])));
  }
}

// NaN-propagating max (torch's amax), and max(m, |a|, |b|) in that sense.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Codes for two values, each returned in the low byte of its word:
// clamp(rint(x*inv), -128, 127).  Adding 1.5*2^23 rounds to the nearest integer
// (ties to even) and leaves it in the low mantissa bits; the lower clamp also
// maps NaN to -128 as fmaxf does in the reference.  No upper clamp is needed:
// |x| <= absmax and inv = 1/(sqrt(G)*scale) with scale >= absmax/(127*sqrt(G))
// bound x*inv by 127*(1+2^-22), which rounds to 127.  The clamp also keeps the
// multiply and the add apart: with nothing between them ptxas fuses the f32x2
// mul.rn and add.rn into one fma, which rounds once and differs at exact ties.
__device__ __forceinline__ uint2 code_bits2(float2 x, float2 inv2) {
  float2 t = mul2(x, inv2);
  t.x = fmaxf(t.x, -128.0f);
  t.y = fmaxf(t.y, -128.0f);
  t = add2(t, make_float2(12582912.0f, 12582912.0f));
  return make_uint2(__float_as_uint(t.x), __float_as_uint(t.y));
}

__device__ __forceinline__ uint32_t pack4(uint2 a, uint2 b) {
  return __byte_perm(__byte_perm(a.x, a.y, 0x0040), __byte_perm(b.x, b.y, 0x0040), 0x5410);
}

// Codes of a row whose rotated values are all finite (no clamp needed, see
// code_bits2): rint(x*inv) as one f32x2 fma with 1.5*2^23, the product not
// rounded on its own, so a product within an fp32 ulp of a half-integer can
// round the other way than code_bits2's.
__device__ __forceinline__ uint2 code_bits2_fused(float2 x, float2 inv2) {
  const float2 t = fma2(x, inv2, make_float2(12582912.0f, 12582912.0f));
  return make_uint2(__float_as_uint(t.x), __float_as_uint(t.y));
}

// Four codes of positions 4w..4w+3 (pairs a = (4w, 4w+1), b = (4w+2, 4w+3))
// packed in reverse: byte 0 is position 4w+3.
__device__ __forceinline__ uint32_t pack4_rev(uint2 a, uint2 b) {
  return pack4(make_uint2(b.y, b.x), make_uint2(a.y, a.x));
}

// The row scale max(am / (127 sqrt(G)), 1e-30) for a finite am >= 0, equal to
// the IEEE quotient the reference divides (int8_convrot.py:95) without a
// division: q = am * RN(1/d), the remainder am - q*d exact in one fma, and one
// fma correction q + rem * RN(1/d) (Markstein's method, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990).  Checked against the division for every non-negative
// finite fp32 and each d = 127 sqrt(G) of G = 4, 16, 64, 256; the quotients
// that the correction can miss are subnormal, below the 1e-30 clamp.
template <int NST>
__device__ __forceinline__ float rot_scale(float am) {
  constexpr float d = 127.0f * float(1 << NST);
  constexpr float c = 1.0f / d;
  const float q = __fmul_rn(am, c);
  const float r = __fmaf_rn(-q, d, am);
  return fmaxf(__fmaf_rn(r, c, q), 1e-30f);
}

template <bool FUSED>
__device__ __forceinline__ uint2 codes2(float2 x, float2 inv2) {
  return FUSED ? code_bits2_fused(x, inv2) : code_bits2(x, inv2);
}

// Codes of one line in output order from the short order's reversed
// positions.  NST == 4: vp is spent and w2[c][jp] holds positions
// c*64 + 16*qd + 2*jp + {0, 1} of the group (qd: the thread's column block),
// i.e. outputs (3-c)*64 + 16*(3-qd) + 15 - 2*jp - {0, 1}; qp points at the
// output block 16*(3-qd) of the group and output quarter r comes from c = 3-r.
// NST < 4: position p of the line holds output p ^ (G - 1), so output word w
// (outputs 4w..4w+3) is position word w ^ ((G - 1) >> 2), bytes reversed.
template <int NST, bool FUSED>
__device__ __forceinline__ void store_codes_short(int8_t* qp, const float2 (&vp)[32], const float2 (&w2)[4][8],
                                                  float2 inv2) {
  if (NST == 4) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int c = 3 - r;
      uint32_t wd[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        wd[k] = pack4_rev(codes2<FUSED>(w2[c][6 - 2 * k], inv2), codes2<FUSED>(w2[c][7 - 2 * k], inv2));
      *reinterpret_cast<uint4*>(qp + r * 64) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    }
  } else {
    constexpr int XW = ((1 << (2 * NST)) - 1) >> 2;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t wd[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int pw = (4 * c + k) ^ XW;
        wd[k] = pack4_rev(codes2<FUSED>(vp[2 * pw], inv2), codes2<FUSED>(vp[2 * pw + 1], inv2));
      }
      *reinterpret_cast<uint4*>(qp + c * 16) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    }
  }
}

// Codes of the rotation-free branch: int8(clamp(round(dtype(v / d)), -128, 127))
// with d the scale rounded to x's dtype, the division IEEE fp32 (torch's
// op-math), dtype() rounding to x's dtype, round() half to even, clamp keeping
// NaN and the int8 cast of NaN giving 0.  Returned in the low byte of a word.
//
// General form, for rows whose d is 0 (fp16 underflow: 0/0 is NaN), inf or NaN.
template <bool BF16>
__device__ __forceinline__ uint32_t rowwise_code(float v, float d) {
  const float t = round_to_dtype<BF16>(__fdiv_rn(v, d));
  const float r = rintf(t);
  if (r != r) return 0u;
  return uint32_t(int(fminf(fmaxf(r, -128.0f), 127.0f)));
}

// Fast form for a finite, non-zero d, four values at a time (a.x, a.y, b.x,
// b.y -> bytes 0..3).  The quotient: q0 = RN(v * rcp) with rcp = RN(1/d) is
// within one ulp of v/d, the remainder v - q0*d is exact as one FMA, and
// RN(q0 + rem * rcp) is the correctly rounded v/d (Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990; quotients small enough to underflow give code 0 either
// way).  |v| <= absmax <= 127 d (1 + 2^-8) keeps |q| < 128.5, so no NaN or
// inf occurs.  The packed dtype rounding, then clamp, then round half to even:
// fp16 adds 1536 (spacing 1 in [1024, 2048), so the add is the rounding and
// the low byte of the sum's bits is the code); bf16, whose spacing is too
// coarse for that, rounds in fp32 with 1.5 * 2^23.  Clamping first equals
// torch's round-then-clamp because the bounds are integers.
template <bool BF16>
__device__ __forceinline__ uint32_t rowwise_codes4(float2 a, float2 b, float2 rcp2, float2 nd2) {
  float2 qa = mul2(a, rcp2), qb = mul2(b, rcp2);
  qa = fma2(fma2(qa, nd2, a), rcp2, qa);
  qb = fma2(fma2(qb, nd2, b), rcp2, qb);
  if (BF16) {
    const __nv_bfloat162 lo = __float2bfloat162_rn(-128.0f), hi = __float2bfloat162_rn(127.0f);
    __nv_bfloat162 ha = __float22bfloat162_rn(qa), hb = __float22bfloat162_rn(qb);
    ha = __hmin2(__hmax2(ha, lo), hi);
    hb = __hmin2(__hmax2(hb, lo), hi);
    const float2 magic = make_float2(12582912.0f, 12582912.0f);
    const float2 fa = add2(unpack2_dtype<true>(*reinterpret_cast<const uint32_t*>(&ha)), magic);
    const float2 fb = add2(unpack2_dtype<true>(*reinterpret_cast<const uint32_t*>(&hb)), magic);
    return pack4(make_uint2(__float_as_uint(fa.x), __float_as_uint(fa.y)),
                 make_uint2(__float_as_uint(fb.x), __float_as_uint(fb.y)));
  }
  const __half2 lo = __float2half2_rn(-128.0f), hi = __float2half2_rn(127.0f), magic = __float2half2_rn(1536.0f);
  __half2 ha = __float22half2_rn(qa), hb = __float22half2_rn(qb);
  ha = __hadd2(__hmin2(__hmax2(ha, lo), hi), magic);
  hb = __hadd2(__hmin2(__hmax2(hb, lo), hi), magic);
  return __byte_perm(*reinterpret_cast<const uint32_t*>(&ha), *reinterpret_cast<const uint32_t*>(&hb), 0x6420);
}

template <int NST, bool BF16, int ACT, bool EXACT, int REGS>
__global__ void __maxnreg__(REGS) rotquant_kernel(const __grid_constant__ CUtensorMap tmx,
                                                       const RotQuantParams p) {
  constexpr float kRoot = float(1 << NST);               // sqrt(G)

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  // Launch-constant values, read once (32-bit: the host guarantees
  // M * K / 64 < 2^31, so batch and line indices fit).
  const int stages = p.stages;
  const uint32_t stage_bytes = p.stage_bytes;
  const int R = p.rows_per_batch;
  const int cpr = p.cpr;
  const int K = p.K;
  const int M = int(p.M);
  const int nbatches = int(p.nbatches);
  const int seg = p.seg;
  const int active_threads = p.active;
  const int boxes = p.boxes;
  const int box_lines = p.box_lines;
  int8_t* const qout = p.q;
  float* const sout = p.scale;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(stages) * stage_bytes);
  unsigned* rowmax = reinterpret_cast<unsigned*>(full + stages);  // [3][R] maxima, then [3][R] NaN flags
  // kActLnMod: ln_words(blockDim.x, R) words after the row maxima, 16-byte
  // aligned (an offset from the shared-memory base, so that the compiler keeps
  // shared-memory loads and stores for them).
  float* const ln_area = reinterpret_cast<float*>(
      smem + ((size_t(stages) * stage_bytes + size_t(stages) * 8u + size_t(6 * R) * 4u + 15u) & ~size_t(15)));
  __shared__ int abort_flag;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  if (tid == 0) {
    prefetch_tmap(&tmx);
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  for (int i = tid; i < 6 * R; i += blockDim.x) rowmax[i] = 0u;
  if constexpr (ACT == kActLnMod) {
    // The column sums past a short row's lines are read as zeros, never written.
    for (int i = tid; i < 16 * R; i += blockDim.x) {
      ln_area[blockDim.x + i] = 0.0f;
      ln_area[2 * blockDim.x + 16 * R + i] = 0.0f;
    }
  }
  __syncthreads();
  // Let the next kernel in the stream (the GEMM) be scheduled as SMs free up;
  // it waits for this grid's completion before reading the codes.  Then wait
  // for whatever produced x before the first load.
  pdl_launch_dependents();
  pdl_wait();

  const int first = blockIdx.x;
  const int step = gridDim.x;
  const uint32_t batch_bytes = uint32_t(boxes) * uint32_t(box_lines) * 128u;

  auto issue = [&](int batch, int s) {
    mbar_arrive_expect_tx(&full[s], batch_bytes);
    uint8_t* dst = smem + size_t(s) * stage_bytes;
    const int line0 = batch * active_threads;
    for (int b = 0; b < boxes; ++b)
      tma_load_2d(dst + size_t(b) * box_lines * 128, &tmx, &full[s], 0, line0 + b * box_lines);
  };

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      const int b = first + s * step;
      if (b < nbatches) issue(b, s);
    }
  }

  const bool active = tid < active_threads;
  const int row_local = tid / cpr;
  const int chunk = tid - row_local * cpr;
  // This thread's line in a ring slot: 128 bytes, 16-byte units swizzled by
  // (line & 7) = (lane & 7); folding that into the base turns each unit's
  // address into base ^ (unit * 16).
  const uint32_t line_off = uint32_t(tid) * 128u + (uint32_t(lane & 7) << 4);
  // Exchange area: the warp's own 4 KB of the slot, rows of 80 bytes (lane L
  // writes row L; the reader of quad gq, position qd reads rows 4gq..4gq+3 at
  // column qd).  Per quarter warp, writes hit 16-byte units 5L + b and reads
  // 4gq + 5c + qd (mod 8): eight distinct units each, so no bank conflicts.
  const uint32_t xw_off = uint32_t(warp) * 4096u + uint32_t(lane) * 80u;
  const uint32_t xr_off = uint32_t(warp) * 4096u + uint32_t(lane >> 2) * 320u + uint32_t(lane & 3) * 16u;
  // Codes of this thread: NST == 4 writes one 16-value block per output
  // quarter of its group (stride 64), else its own 64 contiguous values.
  const int code_off = NST == 4 ? (chunk >> 2) * 256 + (chunk & 3) * 16 : chunk * 64;
  // The short order's reversed positions put NST == 4's block at 3 - qd.
  const int code_off_short = NST == 4 ? (chunk >> 2) * 256 + (3 - (chunk & 3)) * 16 : chunk * 64;

  // Row absmax across lanes: with 32 or more lines a row (K >= 2048) a warp
  // holds parts of at most two rows (the row of its lane 0, and the next), so
  // two warp-wide max reductions cover it; shorter rows use shuffles over
  // segments of `seg` lanes.
  const bool two_rows_per_warp = cpr >= 32;
  const bool in_row0 = row_local == (warp * 32) / cpr;

  int s = 0;
  uint32_t parity = 0;
  int rm_cur = 0;  // rowmax slot of this batch (triple-buffered)
  int abort_batch = nbatches;
  for (int batch = first; batch < nbatches; batch += step) {
    abort_batch = batch;
    if (!mbar_wait(&full[s], parity, DEVERR_TMA_TIMEOUT)) abort_flag = 1;
    uint8_t* buf = smem + size_t(s) * stage_bytes;

    // ---- own line (64 values) from the swizzled ring slot ------------------
    float2 vp[32];
    {
      // XOR on the offset (not on a generic pointer) keeps these shared loads.
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(buf + (line_off ^ uint32_t(c << 4)));
        unpack8<BF16, ACT>(w, &vp[4 * c]);
      }
    }
    if constexpr (ACT == kActLnMod) {
      // LayerNorm over the row (no affine), then the modulation, each result in
      // x's dtype as the separate ops would store it: mean and variance in fp32,
      // sums in a fixed order (per line over its 64 values in pairs, then
      // row_total) times RN(1/K), rstd = RN(1 / sqrt(var + eps)),
      // xn = dtype((x - mean) * rstd), y = dtype(dtype(xn * dtype(1 + scale)) + shift).
      // The last three are packed half-precision adds and multiplies: each gives the fp32 result
      // rounded to the dtype, because 24 bits hold the exact product of two
      // 11-bit (or 8-bit) significands and rounding an fp32 sum or product
      // again to a format of at most 11 bits is innocuous (24 >= 2 * 11 + 2).
      float* const part_s = ln_area;
      float* const col_s = part_s + blockDim.x;
      float* const part_q = col_s + 16 * R;
      float* const col_q = part_q + blockDim.x;
      float2 a = vp[0];
#pragma unroll
      for (int k = 1; k < 32; ++k) a = add2(a, vp[k]);
      const float mean =
          __fmul_rn(row_total(part_s, col_s, __fadd_rn(a.x, a.y), active, row_local, chunk, cpr), p.ln_inv_k);
      const float2 neg_mean = make_float2(-mean, -mean);
      float2 sq = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        vp[k] = add2(vp[k], neg_mean);
        sq = fma2(vp[k], vp[k], sq);
      }
      const float var =
          __fmul_rn(row_total(part_q, col_q, __fadd_rn(sq.x, sq.y), active, row_local, chunk, cpr), p.ln_inv_k);
      const float rstd = __frsqrt_rn(__fadd_rn(var, p.ln_eps));
      const float2 rstd2 = make_float2(rstd, rstd);
      // Modulation vector of this row (rows past M, which are never stored,
      // read the last row's).
      const int64_t row64 = int64_t(batch) * R + row_local;
      const int64_t vec = (row64 < p.M ? row64 : p.M - 1) / p.mod_rows;
      const size_t voff = size_t(vec) * size_t(K) + size_t(chunk) * 64u;
      const uint4* scv = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.mod_scale) + voff);
      const uint4* shv = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.mod_shift) + voff);
      const uint32_t one2 = BF16 ? 0x3f803f80u : 0x3c003c00u;  // (1, 1) in the dtype
      if (active) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 sw = __ldg(scv + c);
          const uint4 hw = __ldg(shv + c);
          const uint32_t su[4] = {sw.x, sw.y, sw.z, sw.w};
          const uint32_t hu[4] = {hw.x, hw.y, hw.z, hw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t xn = pack2_dtype<BF16>(mul2(vp[4 * c + i], rstd2));
            const uint32_t y = hadd2_dt<BF16>(hmul2_dt<BF16>(xn, hadd2_dt<BF16>(one2, su[i])), hu[i]);
            vp[4 * c + i] = unpack2_dtype<BF16>(y);
          }
        }
      }
    }
    if (EXACT) {
      if (NST >= 1) stage0_64(vp);
      if (NST >= 2) stage1_64(vp);
      if (NST >= 3) stage2_64(vp);
    } else {
      if (NST >= 1) stage0_64_short(vp);
      if (NST >= 2) stage1_64_short(vp);
      if (NST >= 3) stage2_64_short(vp);
    }

    float amax;
    // Short order: the thread's own values held a NaN.  Its absmax is then
    // taken again with NaN ignored (as the reference's fmaxf does) and the row
    // is flagged so that its codes take the clamped form.
    bool has_nan = false;
    float2 w2[4][8];  // NST == 4 only: [input c][column pair] of this thread's block
    if (NST == 4) {
      // Swap 16-value blocks among the four threads of a group through this
      // warp's (already consumed) slice of the slot, four values of each
      // block per round, so that afterwards each thread holds one 16-wide
      // column block for all four inputs of the last butterfly, in input order.
      __syncwarp();
#pragma unroll
      for (int r = 0; r < 4; ++r) {
#pragma unroll
        for (int b = 0; b < 4; ++b)
          *reinterpret_cast<float4*>(buf + xw_off + b * 16) =
              make_float4(vp[8 * b + 2 * r].x, vp[8 * b + 2 * r].y, vp[8 * b + 2 * r + 1].x, vp[8 * b + 2 * r + 1].y);
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float4 t = *reinterpret_cast<const float4*>(buf + xr_off + c * 80);
          w2[c][2 * r] = make_float2(t.x, t.y);
          w2[c][2 * r + 1] = make_float2(t.z, t.w);
        }
        __syncwarp();
      }
      // The next TMA into this slot must not overtake these generic accesses.
      fence_proxy_async_smem();
      float am4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {
        if (EXACT) {
          bfly4x2(w2[0][jp], w2[1][jp], w2[2][jp], w2[3][jp]);
#pragma unroll
          for (int r = 0; r < 4; ++r) am4[r] = absmax3(am4[r], w2[r][jp].x, w2[r][jp].y);
        } else {
          bfly4x2_short(w2[0][jp], w2[1][jp], w2[2][jp], w2[3][jp]);
#pragma unroll
          for (int r = 0; r < 4; ++r) am4[r] = absmax3_nan(am4[r], w2[r][jp].x, w2[r][jp].y);
        }
      }
      if (EXACT) {
        amax = fmaxf(fmaxf(am4[0], am4[1]), fmaxf(am4[2], am4[3]));
      } else {
        amax = max_nan(max_nan(am4[0], am4[1]), max_nan(am4[2], am4[3]));
        if (amax != amax) {
          has_nan = true;
          amax = 0.0f;
#pragma unroll
          for (int jp = 0; jp < 8; ++jp)
#pragma unroll
            for (int r = 0; r < 4; ++r) amax = absmax3(amax, w2[r][jp].x, w2[r][jp].y);
        }
      }
    } else if (NST == 0) {
      float am4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int i = 0; i < 32; ++i)
        am4[i & 3] = max_nan(max_nan(am4[i & 3], fabsf(vp[i].x)), fabsf(vp[i].y));
      amax = max_nan(max_nan(am4[0], am4[1]), max_nan(am4[2], am4[3]));
    } else {
      float am4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (EXACT) {
#pragma unroll
        for (int i = 0; i < 32; ++i) am4[i & 3] = absmax3(am4[i & 3], vp[i].x, vp[i].y);
        amax = fmaxf(fmaxf(am4[0], am4[1]), fmaxf(am4[2], am4[3]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) am4[i & 3] = absmax3_nan(am4[i & 3], vp[i].x, vp[i].y);
        amax = max_nan(max_nan(am4[0], am4[1]), max_nan(am4[2], am4[3]));
        if (amax != amax) {
          has_nan = true;
          amax = 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) amax = absmax3(amax, vp[i].x, vp[i].y);
        }
      }
    }

    // ---- row absmax -----------------------------------------------------------
    // (NST == 0: a NaN wins; its sign bit is clear after fabsf, so its bit
    // pattern also wins the unsigned atomicMax below.)
    unsigned* rm = rowmax + rm_cur * R;
    unsigned* rf = rowmax + (3 + rm_cur) * R;  // short order: the row held a NaN
    if (two_rows_per_warp) {
      // Non-negative floats order as their bit patterns: one warp-wide integer
      // max per row, the other row's lanes and idle threads contributing 0.
      const unsigned bits = active ? __float_as_uint(amax) : 0u;
      const unsigned m0 = __reduce_max_sync(0xffffffffu, in_row0 ? bits : 0u);
      const unsigned m1 = __reduce_max_sync(0xffffffffu, in_row0 ? 0u : bits);
      if (active && (lane == 0 || chunk == 0)) atomicMax(&rm[row_local], in_row0 ? m0 : m1);
    } else {
      for (int o = 1; o < seg; o <<= 1) {
        const float other = __shfl_xor_sync(0xffffffffu, amax, o);
        amax = NST == 0 ? max_nan(amax, other) : fmaxf(amax, other);
      }
      if (active && (lane & (seg - 1)) == 0) atomicMax(&rm[row_local], __float_as_uint(amax));
    }
    if (!EXACT && NST != 0 && active && has_nan) atomicOr(&rf[row_local], 1u);
    __syncthreads();
    if (abort_flag) break;

    // Slot s is free again (every thread has read it): refill it.
    if (tid == 0) {
      const int nb = batch + stages * step;
      if (nb < nbatches) issue(nb, s);
    }
    // The slot after next was last read before the previous barrier and is
    // next written after the following one.
    const int rm_clear = rm_cur == 0 ? 2 : rm_cur - 1;
    if (tid < R) {
      rowmax[rm_clear * R + tid] = 0u;
      rowmax[(3 + rm_clear) * R + tid] = 0u;
    }

    const int row = batch * R + row_local;
    if (NST == 0 && active && row < M) {
      // backend.py:230: (amax.float() / 127.0).clamp_min(1e-30); torch divides
      // a CUDA tensor by a host scalar as a multiply by its fp32 reciprocal.
      const float am = __uint_as_float(rm[row_local]);
      float sc = __fmul_rn(am, 1.0f / 127.0f);
      sc = sc != sc ? sc : fmaxf(sc, 1e-30f);
      if (chunk == 0) sout[row] = sc;
      const float d = round_to_dtype<BF16>(sc);  // scale[:, None].to(x.dtype)
      int8_t* qp = qout + size_t(row) * size_t(K) + code_off;
      if (d > 0.0f && d < __int_as_float(0x7f800000)) {  // finite, non-zero
        const float rcp = __frcp_rn(d);
        const float2 rcp2 = make_float2(rcp, rcp), nd2 = make_float2(-d, -d);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t wd[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) wd[k] = rowwise_codes4<BF16>(vp[8 * c + 2 * k], vp[8 * c + 2 * k + 1], rcp2, nd2);
          *reinterpret_cast<uint4*>(qp + c * 16) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t wd[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int i = 8 * c + 2 * k;  // pair index of value 16c + 4k
            wd[k] = pack4(make_uint2(rowwise_code<BF16>(vp[i].x, d), rowwise_code<BF16>(vp[i].y, d)),
                          make_uint2(rowwise_code<BF16>(vp[i + 1].x, d), rowwise_code<BF16>(vp[i + 1].y, d)));
          }
          *reinterpret_cast<uint4*>(qp + c * 16) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
      }
    } else if (NST != 0 && active && row < M) {
      const unsigned am_bits = rm[row_local];
      const float am = __uint_as_float(am_bits);
      const float sc = am_bits < 0x7f800000u ? rot_scale<NST>(am) : am;  // inf stays inf
      if (chunk == 0) sout[row] = sc;
      const float inv = __frcp_rn(__fmul_rn(sc, kRoot));  // correctly rounded: 1 / (sqrt(G) * scale)
      const float2 inv2 = make_float2(inv, inv);
      if (EXACT) {
        int8_t* qp = qout + size_t(row) * size_t(K) + code_off;
        if (NST == 4) {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            uint32_t wd[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
              wd[k] = pack4(code_bits2(w2[r][2 * k], inv2), code_bits2(w2[r][2 * k + 1], inv2));
            *reinterpret_cast<uint4*>(qp + r * 64) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t wd[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int i = 8 * c + 2 * k;  // pair index of value 16c + 4k
              wd[k] = pack4(code_bits2(vp[i], inv2), code_bits2(vp[i + 1], inv2));
            }
            *reinterpret_cast<uint4*>(qp + c * 16) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
          }
        }
      } else {
        // Positions hold outputs in reverse (see bfly4x2_short).  NST == 4:
        // this thread's block (column block qd of input c) holds outputs of
        // block 3 - qd of output quarter 3 - c, each 16 reversed.  NST < 4:
        // position p of the line holds output p ^ (G - 1).
        int8_t* qp = qout + size_t(row) * size_t(K) + code_off_short;
        const bool finite_row = am_bits < 0x7f800000u && rf[row_local] == 0u;
        if (finite_row)
          store_codes_short<NST, true>(qp, vp, w2, inv2);
        else
          store_codes_short<NST, false>(qp, vp, w2, inv2);
      }
    }
    rm_cur = rm_cur == 2 ? 0 : rm_cur + 1;
    if (++s == stages) {
      s = 0;
      parity ^= 1u;
    }
  }

  // A wait gave up: let the copies still in flight land before the CTA exits.
  // The loop left at a batch whose slot s (phase `parity`) is next; the loads
  // in flight are that batch's and the following stages - 1 batches' (slots
  // s, s+1, ... wrapping to the other phase).
  if (abort_flag && tid == 0) {
    for (int k = 0; k < stages; ++k) {
      const int slot = (s + k) % stages;
      const uint32_t par = (s + k < stages) ? parity : (parity ^ 1u);
      if (abort_batch + k * step < nbatches) mbar_wait(&full[slot], par, DEVERR_TMA_TIMEOUT);
    }
  }
}

}  // namespace tg
