/*
 * CPU oracle for the int8_convrot hot path.  TEST INFRASTRUCTURE ONLY: it is the
 * checker that the CUDA kernels are compared against, and the CPU baseline that
 * bench.py times.  The product path never calls it.
 *
 * Three functions, each a plain-C restatement of the reference's algorithm
 * (plus oracle_rotate_quant_short, the kernels' default butterfly order,
 * described where it is defined):
 *
 *  oracle_rotate_quant  - tilegen/kernels/int8_convrot.py:47-104 (`fht_quant`):
 *      per 256-wide group, four radix-4 butterfly stages on the (non-Sylvester)
 *      H4 of tilegen/kernels/hadamard.py:15, stage s at stride 4^s, each output
 *      evaluated left to right exactly as written at int8_convrot.py:74-77;
 *      row absmax; scale = max(absmax / (127*sqrt(G)), 1e-30)  (2032 for G=256,
 *      :95); inv = 1 / (scale * sqrt(G)) (:98); q = clamp(rint(v*inv), -128, 127)
 *      (:100-102).  Generalised to the other powers of four the eager path
 *      accepts (hadamard.py:18-22): G = 4, 16, 64 run 1, 2, 3 stages.  Input is
 *      read exactly into fp32 (fp16 and bf16 upcast without loss, which is what
 *      `_eager_quantize(x.float(), G)` at int8_convrot.py:289-302 sees).
 *
 *  oracle_int8_gemm_dequant - tilegen/quant/int8_ops.py:22-70:
 *      acc = xq @ wq^T in exact int32 (torch._int_mm, :13-19, :62), then
 *      out = ((float(acc) * xscale[m]) * wscale[n]) + bias[n] in fp32, one
 *      rounding per operation, no fused multiply-add (:63-68), then cast to the
 *      output dtype with round-to-nearest-even (`copy_`, :68).
 *
 *  oracle_rowwise_quant - tilegen/comfyui/backend.py:230-232, the
 *      rotation-free branch, as torch evaluates it on CUDA for an fp16/bf16
 *      x: absmax in x's dtype (exact; NaN propagates as torch's amax does),
 *      .float() / 127.0 (a tensor divided by a host scalar: multiplied by the
 *      fp32 reciprocal of 127), clamp_min(1e-30) (NaN kept); divisor
 *      d = scale rounded to x's dtype; q = x / d in fp32 (IEEE) rounded to x's
 *      dtype, round half to even, clamp to [-128, 127] (NaN kept), int8 cast
 *      (NaN -> 0).
 *
 *  oracle_ln_mod - the DiT block's LayerNorm (no affine) and modulation in front
 *      of a projection, y = LN(x) * (1 + scale) + shift, as the CUDA kernel's
 *      fused prologue evaluates it (no reference counterpart: the reference's
 *      path starts at int8_linear's input).  Defined where it is.
 *
 * Build with -ffp-contract=off: a contracted a*b+c would change the rounding.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400u));
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + (127 - 15)) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* fp32 -> fp16, round to nearest even, overflow to inf, NaN kept quiet. */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf or NaN */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477ff000u) { /* >= 65520 rounds to inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx < 0x38800000u) { /* below the smallest fp16 normal: subnormal or 0 */
        /* value = absx as float; fp16 subnormal unit is 2^-24 */
        float a;
        memcpy(&a, &absx, 4);
        /* a * 2^24 rounded to nearest even integer gives the subnormal mantissa */
        float scaled = a * 16777216.0f; /* exact: power-of-two scaling */
        float r = nearbyintf(scaled);
        return (uint16_t)(sign | (uint16_t)r);
    }
    uint32_t exp = (absx >> 23) - 127 + 15;
    uint32_t man = absx & 0x7fffffu;
    uint32_t h = (exp << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* carry may bump exponent: correct */
    return (uint16_t)(sign | h);
}

/* fp32 -> bf16, round to nearest even, NaN kept quiet. */
static uint16_t f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7fffu + lsb;
    return (uint16_t)(x >> 16);
}

static float load_elem(const void *x, int dtype, int64_t i) {
    switch (dtype) {
    case DT_F16: return f16_to_f32(((const uint16_t *)x)[i]);
    case DT_BF16: return bf16_to_f32(((const uint16_t *)x)[i]);
    default: return ((const float *)x)[i];
    }
}

static int group_stages(int group) {
    switch (group) {
    case 4: return 1;
    case 16: return 2;
    case 64: return 3;
    case 256: return 4;
    default: return -1;
    }
}

/* One group, in place: the radix-4 stages of int8_convrot.py:62-80. */
static void rotate_group(float *grp, int group, int nst) {
    for (int st = 0; st < nst; ++st) {
        const int stride = 1 << (2 * st);
        for (int b = 0; b < group / 4; ++b) {
            const int low = b % stride;
            const int high = b / stride;
            const int base = high * 4 * stride + low;
            const float a0 = grp[base];
            const float a1 = grp[base + stride];
            const float a2 = grp[base + 2 * stride];
            const float a3 = grp[base + 3 * stride];
            grp[base] = a0 + a1 + a2 - a3;
            grp[base + stride] = a0 + a1 - a2 + a3;
            grp[base + 2 * stride] = a0 - a1 + a2 + a3;
            grp[base + 3 * stride] = -a0 + a1 + a2 + a3;
        }
    }
}

/* Returns 0 on success, -1 on an unsupported group or a K not divisible by it.
 * Rows are independent; the rotation is computed twice per row (once for the
 * absmax, once for the codes) so that no K-sized scratch is needed. */
int oracle_rotate_quant(const void *x, int dtype, int64_t M, int64_t K, int group,
                        int8_t *q, float *scale) {
    const int nst = group_stages(group);
    if (nst < 0 || K <= 0 || K % group) return -1;
    /* sqrt(G) is a power of two for G a power of four, so the 1/sqrt(G)
     * normalisation folds into one constant exactly as 2032 = 16*127 does for
     * G=256 (int8_convrot.py:93-98). */
    const float root = (float)(1 << nst);
    const float qmax_root = 127.0f * root;
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        float grp[256];
        float amax = 0.0f;
        for (int64_t g0 = 0; g0 < K; g0 += group) {
            for (int i = 0; i < group; ++i) grp[i] = load_elem(x, dtype, m * K + g0 + i);
            rotate_group(grp, group, nst);
            for (int i = 0; i < group; ++i) amax = fmaxf(amax, fabsf(grp[i]));
        }
        const float s = fmaxf(amax / qmax_root, 1e-30f);
        scale[m] = s;
        const float inv = 1.0f / (s * root);
        for (int64_t g0 = 0; g0 < K; g0 += group) {
            for (int i = 0; i < group; ++i) grp[i] = load_elem(x, dtype, m * K + g0 + i);
            rotate_group(grp, group, nst);
            for (int i = 0; i < group; ++i) {
                float v = nearbyintf(grp[i] * inv);
                v = fminf(fmaxf(v, -128.0f), 127.0f);
                q[m * K + g0 + i] = (int8_t)v;
            }
        }
    }
    return 0;
}

/* The kernel's default ("short") butterfly order, restated: per radix-4
 * butterfly S = (a0 + a2) + (a1 + a3) and output 3 - i = fma(-2, a_i, S) --
 * the same H4 (every row all ones but a single -1) with fewer roundings.  Not
 * the reference's order: parity with the reference is the north-star
 * tolerance (codes +-1 on <= 0.1 %, scales 1e-3 relative), checked in the
 * tests against oracle_rotate_quant and the golden vectors. */
static void rotate_group_short(float *grp, int group, int nst) {
    for (int st = 0; st < nst; ++st) {
        const int stride = 1 << (2 * st);
        for (int b = 0; b < group / 4; ++b) {
            const int low = b % stride;
            const int high = b / stride;
            const int base = high * 4 * stride + low;
            const float a0 = grp[base];
            const float a1 = grp[base + stride];
            const float a2 = grp[base + 2 * stride];
            const float a3 = grp[base + 3 * stride];
            const float s = (a0 + a2) + (a1 + a3);
            grp[base] = fmaf(-2.0f, a3, s);
            grp[base + stride] = fmaf(-2.0f, a2, s);
            grp[base + 2 * stride] = fmaf(-2.0f, a1, s);
            grp[base + 3 * stride] = fmaf(-2.0f, a0, s);
        }
    }
}

/* Rotate+quant in the short order.  Scale as oracle_rotate_quant (absmax with
 * NaN ignored).  Codes of a row whose rotated values are all finite:
 * rint(v * inv) of the exact product (one fma with 1.5 * 2^23, as the kernel
 * does); any other row: clamp(rint(v * inv)) with the product rounded first
 * and NaN -> -128, as oracle_rotate_quant. */
int oracle_rotate_quant_short(const void *x, int dtype, int64_t M, int64_t K, int group,
                              int8_t *q, float *scale) {
    const int nst = group_stages(group);
    if (nst < 0 || K <= 0 || K % group) return -1;
    const float root = (float)(1 << nst);
    const float qmax_root = 127.0f * root;
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        float grp[256];
        float amax = 0.0f;
        int finite = 1;
        for (int64_t g0 = 0; g0 < K; g0 += group) {
            for (int i = 0; i < group; ++i) grp[i] = load_elem(x, dtype, m * K + g0 + i);
            rotate_group_short(grp, group, nst);
            for (int i = 0; i < group; ++i) {
                amax = fmaxf(amax, fabsf(grp[i]));
                if (!isfinite(grp[i])) finite = 0;
            }
        }
        const float s = fmaxf(amax / qmax_root, 1e-30f);
        scale[m] = s;
        const float inv = 1.0f / (s * root);
        for (int64_t g0 = 0; g0 < K; g0 += group) {
            for (int i = 0; i < group; ++i) grp[i] = load_elem(x, dtype, m * K + g0 + i);
            rotate_group_short(grp, group, nst);
            for (int i = 0; i < group; ++i) {
                float v;
                if (finite) {
                    v = fmaf(grp[i], inv, 12582912.0f) - 12582912.0f;
                } else {
                    v = nearbyintf(grp[i] * inv);
                    v = fminf(fmaxf(v, -128.0f), 127.0f);
                }
                q[m * K + g0 + i] = (int8_t)v;
            }
        }
    }
    return 0;
}

static float round_to_dtype(float v, int dtype) {
    return dtype == DT_BF16 ? bf16_to_f32(f32_to_bf16(v)) : f16_to_f32(f32_to_f16(v));
}

/* Sum of one row's per-line partials part[0..lines) in the kernel's fixed
 * order: column c < 16 adds lines c, c + 16, c + 32, ... ascending (columns
 * past the lines are 0), then the 16 columns are added as a pairwise tree,
 * ((c0 + c1) + (c2 + c3)) + ((c4 + c5) + (c6 + c7)) + ... . */
static float ln_row_total(const float *part, int lines) {
    float col[16];
    for (int c = 0; c < 16; ++c) {
        if (c >= lines) {
            col[c] = 0.0f;
            continue;
        }
        float t = part[c];
        for (int l = c + 16; l < lines; l += 16) t += part[l];
        col[c] = t;
    }
    float q[4];
    for (int i = 0; i < 4; ++i) q[i] = (col[4 * i] + col[4 * i + 1]) + (col[4 * i + 2] + col[4 * i + 3]);
    return (q[0] + q[1]) + (q[2] + q[3]);
}

/* 1 / sqrt(v) rounded to the nearest float (ties to even), as the kernel's
 * correctly rounded reciprocal square root: a candidate from double
 * precision, then the exact side of each neighbouring midpoint m from the sign
 * of m*m*v - 1 (m*m is exact in double; one fma rounds the rest once, which
 * keeps the sign). */
static uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static float rsqrt_rn(float v) {
    if (isnan(v) || v < 0.0f) return NAN;
    if (v == 0.0f) return signbit(v) ? -INFINITY : INFINITY;
    if (isinf(v)) return 0.0f;
    float f = (float)(1.0 / sqrt((double)v));
    for (int it = 0; it < 2; ++it) {
        const float up = nextafterf(f, INFINITY);
        const double mu = ((double)f + (double)up) * 0.5;
        const double su = fma(mu * mu, (double)v, -1.0);  /* < 0: 1/sqrt(v) above the midpoint */
        if (su < 0.0 || (su == 0.0 && (f32_bits(up) & 1u) == 0u)) {
            f = up;
            continue;
        }
        const float dn = nextafterf(f, 0.0f);
        const double md = ((double)f + (double)dn) * 0.5;
        const double sd = fma(md * md, (double)v, -1.0);  /* > 0: 1/sqrt(v) below the midpoint */
        if (sd > 0.0 || (sd == 0.0 && (f32_bits(dn) & 1u) == 0u)) {
            f = dn;
            continue;
        }
        break;
    }
    return f;
}

/* y = dtype(dtype(dtype((x - mean) * rstd) * dtype(1 + scale[v])) + shift[v])
 * for row m and v = m / mod_rows, with, per row of K = 64 * lines values:
 *   line sums: pairs (2k, 2k+1) of the line's 64 values accumulated in two
 *     lanes, k ascending, then lane 0 + lane 1; mean = total(line sums) * RN(1/K);
 *   d = x - mean; line sums of squares the same way with fmaf(d, d, acc);
 *   var = total * RN(1/K); rstd = 1 / sqrt(var + eps) correctly rounded;
 * every operation in fp32 rounded once, then each named rounding to the dtype.
 * x, scale, shift, y hold raw fp16/bf16 patterns ([M][K], [.][K], [.][K], [M][K]).
 * Returns 0 on success, -1 on a bad argument. */
int oracle_ln_mod(const uint16_t *x, int dtype, int64_t M, int64_t K, float eps, const uint16_t *scale,
                  const uint16_t *shift, int64_t mod_rows, uint16_t *y) {
    if ((dtype != DT_F16 && dtype != DT_BF16) || K <= 0 || K % 64 != 0 || K / 64 > 1024 || M < 0 ||
        mod_rows < 1)
        return -1;
    const int lines = (int)(K / 64);
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        float part[1024];
        float d[64];
        const int64_t v = m / mod_rows;
        for (int l = 0; l < lines; ++l) {
            float a0 = 0.0f, a1 = 0.0f;
            for (int k = 0; k < 32; ++k) {
                const float e0 = load_elem(x, dtype, m * K + l * 64 + 2 * k);
                const float e1 = load_elem(x, dtype, m * K + l * 64 + 2 * k + 1);
                a0 = k == 0 ? e0 : a0 + e0;
                a1 = k == 0 ? e1 : a1 + e1;
            }
            part[l] = a0 + a1;
        }
        const float inv_k = 1.0f / (float)K;
        const float mean = ln_row_total(part, lines) * inv_k;
        for (int l = 0; l < lines; ++l) {
            float q0 = 0.0f, q1 = 0.0f;
            for (int k = 0; k < 32; ++k) {
                const float d0 = load_elem(x, dtype, m * K + l * 64 + 2 * k) - mean;
                const float d1 = load_elem(x, dtype, m * K + l * 64 + 2 * k + 1) - mean;
                q0 = fmaf(d0, d0, q0);
                q1 = fmaf(d1, d1, q1);
            }
            part[l] = q0 + q1;
        }
        const float var = ln_row_total(part, lines) * inv_k;
        const float rstd = rsqrt_rn(var + eps);
        for (int l = 0; l < lines; ++l) {
            for (int j = 0; j < 64; ++j) d[j] = load_elem(x, dtype, m * K + l * 64 + j) - mean;
            for (int j = 0; j < 64; ++j) {
                const int64_t c = (int64_t)l * 64 + j;
                const float xn = round_to_dtype(d[j] * rstd, dtype);
                const float t1 = round_to_dtype(1.0f + load_elem(scale, dtype, v * K + c), dtype);
                const float pr = round_to_dtype(xn * t1, dtype);
                const float out = pr + load_elem(shift, dtype, v * K + c);
                y[m * K + c] = dtype == DT_BF16 ? f32_to_bf16(out) : f32_to_f16(out);
            }
        }
    }
    return 0;
}

/* Returns 0 on success, -1 on a bad argument (dtype must be DT_F16 or DT_BF16). */
int oracle_rowwise_quant(const void *x, int dtype, int64_t M, int64_t K, int8_t *q, float *scale) {
    if ((dtype != DT_F16 && dtype != DT_BF16) || K <= 0 || M < 0) return -1;
    const float inv127 = 1.0f / 127.0f;
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        float amax = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float a = fabsf(load_elem(x, dtype, m * K + k));
            if (isnan(a) || isnan(amax)) amax = NAN;
            else if (a > amax) amax = a;
        }
        float s = amax * inv127;
        if (!isnan(s) && s < 1e-30f) s = 1e-30f;
        scale[m] = s;
        const float d = round_to_dtype(s, dtype);
        for (int64_t k = 0; k < K; ++k) {
            const float t = round_to_dtype(load_elem(x, dtype, m * K + k) / d, dtype);
            float r = nearbyintf(t);
            if (isnan(r)) {
                q[m * K + k] = 0;
                continue;
            }
            r = fminf(fmaxf(r, -128.0f), 127.0f);
            q[m * K + k] = (int8_t)r;
        }
    }
    return 0;
}

/* Returns 0 on success, -1 on a bad argument.  wscale_numel is 1 (a scalar
 * broadcast, int8_ops.py:49-53) or N.  bias may be NULL.  out_dtype is one of
 * DT_F32, DT_F16, DT_BF16. */
int oracle_int8_gemm_dequant(const int8_t *xq, const float *xscale, const int8_t *wq,
                             const float *wscale, int64_t wscale_numel, const float *bias,
                             int64_t M, int64_t N, int64_t K, int out_dtype, void *out) {
    if (M < 0 || N <= 0 || K <= 0) return -1;
    if (wscale_numel != 1 && wscale_numel != N) return -1;
    if (out_dtype != DT_F32 && out_dtype != DT_F16 && out_dtype != DT_BF16) return -1;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t m = 0; m < M; ++m) {
        const int8_t *a = xq + m * K;
        const float xs = xscale[m];
        for (int64_t n = 0; n < N; ++n) {
            const int8_t *b = wq + n * K;
            int32_t acc = 0;
            for (int64_t k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
            float v = (float)acc;          /* int32 -> fp32, round to nearest */
            v = v * xs;
            v = v * wscale[wscale_numel == 1 ? 0 : n];
            if (bias) v = v + bias[n];
            const int64_t o = m * N + n;
            if (out_dtype == DT_F32) ((float *)out)[o] = v;
            else if (out_dtype == DT_F16) ((uint16_t *)out)[o] = f32_to_f16(v);
            else ((uint16_t *)out)[o] = f32_to_bf16(v);
        }
    }
    return 0;
}

/* Threads the oracle will use (OpenMP), for the CPU-baseline report. */
int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
