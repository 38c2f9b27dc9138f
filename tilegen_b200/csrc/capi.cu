// Host side of the tilegen_b200 C ABI (include/tilegen_b200.h): argument
// checks, launch-shape selection, TMA descriptor encoding and the launches.
// One translation unit holds every kernel so they share the device status word.
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "gemm_i8.cuh"
#include "gemm_splitk.cuh"
#include "gemv_i8.cuh"
#include "rotquant.cuh"

namespace {

constexpr int kMaxDevices = 64;
constexpr int64_t kRotQuantMaxK = 32768;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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

struct DeviceInfo {
  int sms = 0;       // SMs the persistent kernels may use (the SM budget applied)
  int sms_all = 0;   // SMs of the device
};

// Process-wide cap on the SMs the persistent kernels (rotate+quant, the tiled
// GEMM) size their grids for; 0 = every SM (tg_set_sm_budget).
std::atomic<int> g_sm_budget{0};

bool current_device(int* dev, DeviceInfo* info) {
  static DeviceInfo cache[kMaxDevices];
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= kMaxDevices) return false;
  if (cache[*dev].sms == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, *dev) != cudaSuccess) return false;
    cache[*dev].sms = v;
    cache[*dev].sms_all = v;
  }
  *info = cache[*dev];
  const int budget = g_sm_budget.load(std::memory_order_relaxed);
  if (budget > 0 && budget < info->sms) info->sms = budget;
  return true;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D tiled tensor map, innermost dimension first.
bool make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per-(kernel, device) one-time attribute setup.
template <typename K>
bool ensure_smem_attr(K kernel, int dev, uint32_t bytes, uint32_t* done_bytes) {
  if (done_bytes[dev] >= bytes) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)) != cudaSuccess)
    return false;
  done_bytes[dev] = bytes;
  return true;
}

// ------------------------------------------------------------------ rotate+quant
// Dynamic shared memory of a launch: alignment slack, the ring of `stages`
// slots, their mbarriers, the row maxima and NaN flags ([3][R] each), and for
// the LayerNorm prologue its partial sums (the CTA has stage_bytes / 128 threads).
uint32_t rotquant_smem(int stages, uint32_t stage_bytes, int R, bool ln) {
  const uint32_t ln_bytes = ln ? uint32_t(tg::ln_words(int(stage_bytes / 128u), R)) * 4u : 0u;
  return 1024u + uint32_t(stages) * stage_bytes + uint32_t(stages) * 8u + uint32_t(6 * R) * 4u + ln_bytes;
}

constexpr uint32_t kSmemPerCtaMax = 232448u;  // 227 KB: the opt-in maximum of one CTA
constexpr uint32_t kSmemPerSm = 233472u;      // 228 KB per SM, 1 KB of it reserved per resident CTA

// CTAs per SM that a rotquant variant's registers allow (with the shallowest
// ring), and the deepest ring (2 to 4 slots) that that many CTAs fit.
template <int NST, bool BF16, int ACT, bool EXACT, int REGS>
bool rotquant_shape(int dev, int threads, uint32_t stage_bytes, int R, int* occ_out, int* stages_out) {
  static uint32_t attr_done[kMaxDevices];
  static uint32_t static_smem = ~0u;
  // (occ | stages << 8) per device, CTA width in warps and rows per batch; 0 = not known yet.
  static int known[kMaxDevices][17][9];
  const int tw = threads / 32;
  if (tw <= 16 && R <= 8 && known[dev][tw][R] != 0) {
    *occ_out = known[dev][tw][R] & 0xff;
    *stages_out = known[dev][tw][R] >> 8;
    return true;
  }
  auto kern = tg::rotquant_kernel<NST, BF16, ACT, EXACT, REGS>;
  if (static_smem == ~0u) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return false;
    static_smem = uint32_t(fa.sharedSizeBytes);
  }
  const uint32_t dyn_max = kSmemPerCtaMax - static_smem;  // static + dynamic <= the per-CTA maximum
  if (!ensure_smem_attr(kern, dev, dyn_max, attr_done)) return false;
  int occ = 0;
  constexpr bool kLn = ACT == tg::kActLnMod;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, rotquant_smem(2, stage_bytes, R, kLn)) !=
          cudaSuccess ||
      occ < 1)
    return false;
  int stages = 4;
  while (stages > 2 && (rotquant_smem(stages, stage_bytes, R, kLn) > dyn_max ||
                        uint64_t(occ) * (rotquant_smem(stages, stage_bytes, R, kLn) + static_smem + 1024u) >
                            kSmemPerSm))
    --stages;
  *occ_out = occ;
  *stages_out = stages;
  if (tw <= 16 && R <= 8) known[dev][tw][R] = occ | (stages << 8);
  return true;
}

template <int NST, bool BF16, int ACT, bool EXACT, int REGS>
int launch_rotquant_t(const CUtensorMap& tm, tg::RotQuantParams p, int threads, int occ, int dev, int sms,
                      cudaStream_t st) {
  auto kern = tg::rotquant_kernel<NST, BF16, ACT, EXACT, REGS>;
  const uint32_t smem = rotquant_smem(p.stages, p.stage_bytes, p.rows_per_batch, ACT == tg::kActLnMod);
  const int64_t grid64 = std::min<int64_t>(p.nbatches, int64_t(sms) * occ);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(unsigned(grid64));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, tm, p) != cudaSuccess) return TG_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TG_OK : TG_ERR_CUDA;
}

// The register budget.  96 registers a thread by default; the hot form (G=256,
// short order, no activation) also has an 80-register build, taken when it
// keeps more warps resident: a CTA of seven warps (K=13824: 216 lines a row)
// fits twice per SM at 96 registers (five warps' registers per SM
// sub-partition) but three times at 80.
template <int NST, bool BF16, int ACT, bool EXACT>
int launch_rotquant_regs(const CUtensorMap& tm, tg::RotQuantParams p, int threads, int dev, int sms,
                         cudaStream_t st) {
  int occ = 0, stages = 0;
  if (!rotquant_shape<NST, BF16, ACT, EXACT, 96>(dev, threads, p.stage_bytes, p.rows_per_batch, &occ, &stages))
    return TG_ERR_CUDA;
  if constexpr (NST == 4 && ACT == tg::kActNone && !EXACT) {
    int occ80 = 0, stages80 = 0;
    if (!rotquant_shape<NST, BF16, ACT, EXACT, 80>(dev, threads, p.stage_bytes, p.rows_per_batch, &occ80,
                                                   &stages80))
      return TG_ERR_CUDA;
    if (occ80 > occ) {
      p.stages = stages80;
      return launch_rotquant_t<NST, BF16, ACT, EXACT, 80>(tm, p, threads, occ80, dev, sms, st);
    }
  }
  p.stages = stages;
  return launch_rotquant_t<NST, BF16, ACT, EXACT, 96>(tm, p, threads, occ, dev, sms, st);
}

// Internal code of the LayerNorm + modulation prologue (tg_quantize_ln_mod),
// beside the public TG_ACT_* codes.
constexpr int kLnModCode = 3;

template <int NST, bool BF16, bool EXACT>
int launch_rotquant_act(int act, const CUtensorMap& tm, const tg::RotQuantParams& p, int threads, int dev, int sms,
                        cudaStream_t st) {
  switch (act) {
    case TG_ACT_GELU_TANH:
      return launch_rotquant_regs<NST, BF16, tg::kActGeluTanh, EXACT>(tm, p, threads, dev, sms, st);
    case TG_ACT_GELU: return launch_rotquant_regs<NST, BF16, tg::kActGelu, EXACT>(tm, p, threads, dev, sms, st);
    case kLnModCode:
      // Built for the rotated groups in the short order only.
      if constexpr (NST > 0 && !EXACT) {
        return launch_rotquant_regs<NST, BF16, tg::kActLnMod, EXACT>(tm, p, threads, dev, sms, st);
      } else {
        return TG_ERR_UNSUPPORTED;
      }
    default: return launch_rotquant_regs<NST, BF16, tg::kActNone, EXACT>(tm, p, threads, dev, sms, st);
  }
}

// The butterfly order: the reference kernel's (bit-identical to it) or the
// short one (the default).  The rotation-free form has no butterflies.
template <int NST, bool BF16>
int launch_rotquant_order(bool exact, int act, const CUtensorMap& tm, const tg::RotQuantParams& p, int threads,
                          int dev, int sms, cudaStream_t st) {
  if constexpr (NST == 0) {
    return launch_rotquant_act<NST, BF16, true>(act, tm, p, threads, dev, sms, st);
  } else {
    if (exact) return launch_rotquant_act<NST, BF16, true>(act, tm, p, threads, dev, sms, st);
    return launch_rotquant_act<NST, BF16, false>(act, tm, p, threads, dev, sms, st);
  }
}

int gcd_int(int a, int b) {
  while (b) {
    const int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

// The LayerNorm + modulation prologue's arguments (tg_quantize_ln_mod).
struct LnModArgs {
  const void* scale;
  const void* shift;
  int64_t rows;
  float eps;
};

// The shared body of tg_quantize_act and tg_quantize_ln_mod: shape checks,
// launch shape, tensor map, launch.
int quantize_launch(const void* x, int x_dtype, int64_t M, int64_t K, int group, int act, bool exact,
                    const LnModArgs* ln, int8_t* q, float* scale, void* stream);

}  // namespace

extern "C" {

int tg_version(void) { return (0 << 16) | 1; }

const char* tg_status_string(int s) {
  switch (s) {
    case TG_OK: return "ok";
    case TG_ERR_INVALID_ARG: return "invalid argument";
    case TG_ERR_UNSUPPORTED: return "unsupported shape or group size";
    case TG_ERR_MISALIGNED: return "pointer not 16-byte aligned";
    case TG_ERR_CUDA: return "CUDA call failed";
    case TG_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait expired";
    default: return "unknown status";
  }
}

int64_t tg_rotate_quant_max_k(void) { return kRotQuantMaxK; }

int tg_rotate_quant(const void* x, int x_dtype, int64_t M, int64_t K, int group, int8_t* q, float* scale,
                    void* stream) {
  if (group == 1) {  // the rotation-free branch is tg_quantize_act's
    if (M < 0 || K <= 0 || (x_dtype != TG_DT_F16 && x_dtype != TG_DT_BF16)) return TG_ERR_INVALID_ARG;
    return TG_ERR_UNSUPPORTED;
  }
  return tg_quantize_act(x, x_dtype, M, K, group, TG_ACT_NONE, q, scale, stream);
}

int tg_quantize_act(const void* x, int x_dtype, int64_t M, int64_t K, int group, int act, int8_t* q, float* scale,
                    void* stream) {
  if (M < 0 || K <= 0) return TG_ERR_INVALID_ARG;
  if (x_dtype != TG_DT_F16 && x_dtype != TG_DT_BF16) return TG_ERR_INVALID_ARG;
  const bool exact = (act & TG_QUANT_REFERENCE_ORDER) != 0;
  act &= ~TG_QUANT_REFERENCE_ORDER;
  if (act != TG_ACT_NONE && act != TG_ACT_GELU_TANH && act != TG_ACT_GELU) return TG_ERR_INVALID_ARG;
  return quantize_launch(x, x_dtype, M, K, group, act, exact, nullptr, q, scale, stream);
}

int tg_quantize_ln_mod(const void* x, int x_dtype, int64_t M, int64_t K, int group, float eps, const void* mod_scale,
                       const void* mod_shift, int64_t mod_rows, int8_t* q, float* scale, void* stream) {
  if (M < 0 || K <= 0 || mod_rows < 1) return TG_ERR_INVALID_ARG;
  if (x_dtype != TG_DT_F16 && x_dtype != TG_DT_BF16) return TG_ERR_INVALID_ARG;
  if (!(eps >= 0.0f) || eps > 3.0e38f) return TG_ERR_INVALID_ARG;  // also rejects NaN
  if (group == 1) return TG_ERR_UNSUPPORTED;                         // rotated groups only
  if (M > 0) {
    if (!mod_scale || !mod_shift) return TG_ERR_INVALID_ARG;
    if (!aligned16(mod_scale) || !aligned16(mod_shift)) return TG_ERR_MISALIGNED;
  }
  const LnModArgs ln{mod_scale, mod_shift, mod_rows, eps};
  return quantize_launch(x, x_dtype, M, K, group, kLnModCode, false, &ln, q, scale, stream);
}

}  // extern "C"

namespace {

int quantize_launch(const void* x, int x_dtype, int64_t M, int64_t K, int group, int act, bool exact,
                    const LnModArgs* ln, int8_t* q, float* scale, void* stream) {
  int nst;
  switch (group) {
    case 1: nst = 0; break;
    case 4: nst = 1; break;
    case 16: nst = 2; break;
    case 64: nst = 3; break;
    case 256: nst = 4; break;
    default: return TG_ERR_UNSUPPORTED;
  }
  // Rotated: K % 256 as the reference launcher requires (int8_convrot.py:196-230).
  // Row-wise: whole 64-element lines (one thread owns one).
  if (K % (nst == 0 ? 64 : 256) != 0 || K > kRotQuantMaxK) return TG_ERR_UNSUPPORTED;
  if (M == 0) return TG_OK;
  if (!x || !q || !scale) return TG_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(q) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return TG_ERR_MISALIGNED;
  const int cpr = int(K / 64);
  // 32-bit line and batch indices in the kernel (with up to 8 rows of slack).
  if ((M + 8) * int64_t(cpr) >= (int64_t(1) << 31)) return TG_ERR_UNSUPPORTED;

  // Rows per batch: the fewest that fill whole warps to within 5 %.
  int R = 1;
  for (int r = 1; r <= 8; ++r) {
    const int lines = r * cpr;
    const int thr = (lines + 31) / 32 * 32;
    if (thr > 512) break;
    if ((thr - lines) * 20 <= lines) {
      R = r;
      break;
    }
  }
  const int active = R * cpr;
  const int threads = (active + 31) / 32 * 32;
  if (threads > 512) return TG_ERR_UNSUPPORTED;
  int box = active;
  if (box > 256) {
    box = 4;
    for (int d = 256; d >= 4; --d)
      if (active % d == 0) {
        box = d;
        break;
      }
  }
  // The ring's depth (2 to 4 slots) is chosen at launch from the kernel's
  // occupancy (launch_rotquant_regs).
  const uint32_t stage_bytes = uint32_t(threads) * 128u;

  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;

  CUtensorMap tm;
  if (!make_tmap_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, x, 64, uint64_t(M) * uint64_t(cpr), 128, 64,
                    uint32_t(box), CU_TENSOR_MAP_SWIZZLE_128B))
    return TG_ERR_CUDA;

  tg::RotQuantParams p;
  p.q = q;
  p.scale = scale;
  p.M = M;
  p.K = int(K);
  p.cpr = cpr;
  p.rows_per_batch = R;
  p.active = active;
  p.box_lines = box;
  p.boxes = active / box;
  p.nbatches = (M + R - 1) / R;
  p.stages = 2;
  p.stage_bytes = stage_bytes;
  p.seg = gcd_int(cpr, 32);
  p.mod_scale = ln ? ln->scale : nullptr;
  p.mod_shift = ln ? ln->shift : nullptr;
  p.mod_rows = ln ? ln->rows : 1;
  p.ln_eps = ln ? ln->eps : 0.0f;
  p.ln_inv_k = 1.0f / float(K);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = x_dtype == TG_DT_BF16;
#define TG_RQ_CASE(N)                                                                           \
  case N:                                                                                       \
    return bf ? launch_rotquant_order<N, true>(exact, act, tm, p, threads, dev, info.sms, st) \
              : launch_rotquant_order<N, false>(exact, act, tm, p, threads, dev, info.sms, st);
  switch (nst) {
    TG_RQ_CASE(0)
    TG_RQ_CASE(1)
    TG_RQ_CASE(2)
    TG_RQ_CASE(3)
    default:
      return bf ? launch_rotquant_order<4, true>(exact, act, tm, p, threads, dev, info.sms, st)
                : launch_rotquant_order<4, false>(exact, act, tm, p, threads, dev, info.sms, st);
  }
#undef TG_RQ_CASE
}

}  // namespace

namespace {

template <int BN, int OUT, bool HAS_BIAS, bool PAIR>
int launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const tg::GemmParams& p,
                  int dev, int units, cudaStream_t st) {
  static uint32_t attr_done[kMaxDevices];
  constexpr uint32_t smem = tg::gemm::smem_bytes(BN, PAIR);
  auto kern = tg::gemm_i8_dequant_kernel<BN, OUT, HAS_BIAS, PAIR>;
  if (!ensure_smem_attr(kern, dev, smem, attr_done)) return TG_ERR_CUDA;
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid_units = tiles < units ? tiles : units;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3(unsigned(grid_units * (PAIR ? 2 : 1)));
  cfg.blockDim = dim3(tg::gemm::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: the prologue overlaps the previous kernel
  // (the quantiser), the kernel waits for it before reading xq/xscale.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, to, p) != cudaSuccess) return TG_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TG_OK : TG_ERR_CUDA;
}

template <int BN, bool PAIR>
int launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const tg::GemmParams& p,
                   int out_dtype, bool has_bias, int dev, int units, cudaStream_t st) {
  switch (out_dtype) {
    case TG_DT_F32: return has_bias ? launch_gemm_t<BN, 0, true, PAIR>(ta, tb, to, p, dev, units, st)
                                    : launch_gemm_t<BN, 0, false, PAIR>(ta, tb, to, p, dev, units, st);
    case TG_DT_F16: return has_bias ? launch_gemm_t<BN, 1, true, PAIR>(ta, tb, to, p, dev, units, st)
                                    : launch_gemm_t<BN, 1, false, PAIR>(ta, tb, to, p, dev, units, st);
    default: return has_bias ? launch_gemm_t<BN, 2, true, PAIR>(ta, tb, to, p, dev, units, st)
                             : launch_gemm_t<BN, 2, false, PAIR>(ta, tb, to, p, dev, units, st);
  }
}

template <bool PAIR>
int launch_gemm_mode(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                     const tg::GemmParams& p, int out_dtype, bool hb, int dev, int units, cudaStream_t st) {
  switch (bn) {
    case 224: return launch_gemm_bn<224, PAIR>(ta, tb, to, p, out_dtype, hb, dev, units, st);
    case 192: return launch_gemm_bn<192, PAIR>(ta, tb, to, p, out_dtype, hb, dev, units, st);
    case 160: return launch_gemm_bn<160, PAIR>(ta, tb, to, p, out_dtype, hb, dev, units, st);
    case 128: return launch_gemm_bn<128, PAIR>(ta, tb, to, p, out_dtype, hb, dev, units, st);
    default: return launch_gemm_bn<256, PAIR>(ta, tb, to, p, out_dtype, hb, dev, units, st);
  }
}

// Tile-processing units that can be resident at once: SMs for single-CTA
// tiles, co-resident clusters of 2 for pair tiles (queried once per device).
int gemm_units(int dev, int sms, bool pair) {
  static int cache[kMaxDevices];
  if (!pair) return sms;
  if (cache[dev] > 0) return cache[dev] < sms / 2 ? cache[dev] : sms / 2;
  int all = sms;
  if (cudaDeviceGetAttribute(&all, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) all = sms;
  auto kern = tg::gemm_i8_dequant_kernel<256, 1, false, true>;
  constexpr uint32_t smem = tg::gemm::smem_bytes(256, true);
  static uint32_t attr_done[kMaxDevices];
  int n = 0;
  if (ensure_smem_attr(kern, dev, smem, attr_done)) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(unsigned(all));
    cfg.blockDim = dim3(tg::gemm::THREADS);
    cfg.dynamicSmemBytes = smem;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cache[dev] = n > 0 ? n : all / 2;
  return cache[dev] < sms / 2 ? cache[dev] : sms / 2;
}

// Tile shape for an M x N problem.  The persistent grid runs
// ceil(tiles / units) waves of tiles costing about (BN + kTileOverhead) column
// steps each; pick the width minimising waves * (BN + overhead).  Pair tiles
// (256 rows on two SMs) are used whenever M has more than one 128-row block.
constexpr int kGemmWidths[] = {256, 224, 192, 160, 128};
constexpr int kTileOverhead = 32;
int g_forced_bn = 0;     // tg_set_gemm_config(): 0 = cost model
int g_forced_pair = -1;  // -1 = by M

void pick_gemm_config(int64_t M, int64_t N, int dev, int sms, int* bn_out, int* pair_out) {
  const bool pair = g_forced_pair >= 0 ? g_forced_pair != 0 : M > tg::gemm::BM;
  const int units = gemm_units(dev, sms, pair);
  const int64_t tm = pair ? 2 * tg::gemm::BM : tg::gemm::BM;
  const int64_t mt = (M + tm - 1) / tm;
  int best = 256;
  int64_t best_cost = -1;
  for (int bn : kGemmWidths) {
    const int64_t tiles = mt * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + units - 1) / units;
    const int64_t cost = waves * (bn + kTileOverhead);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  *bn_out = g_forced_bn ? g_forced_bn : best;
  *pair_out = pair ? 1 : 0;
}

}  // namespace

extern "C" {

int tg_int8_gemm_dequant(const int8_t* xq, const float* xscale, const int8_t* wq, const float* wscale,
                         int64_t wscale_numel, const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K,
                         int out_dtype, void* out, void* stream) {
  using namespace tg::gemm;
  if (M < 0 || N <= 0 || K <= 0) return TG_ERR_INVALID_ARG;
  if (out_dtype != TG_DT_F32 && out_dtype != TG_DT_F16 && out_dtype != TG_DT_BF16) return TG_ERR_INVALID_ARG;
  if (bias && bias_dtype != TG_DT_F32 && bias_dtype != TG_DT_F16 && bias_dtype != TG_DT_BF16)
    return TG_ERR_INVALID_ARG;
  if (wscale_numel != 1 && wscale_numel != N) return TG_ERR_INVALID_ARG;
  const int esz = out_dtype == TG_DT_F32 ? 4 : 2;
  if (K % 16 != 0 || (N * esz) % 16 != 0) return TG_ERR_UNSUPPORTED;
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31)) return TG_ERR_UNSUPPORTED;
  if (M == 0) return TG_OK;
  if (!xq || !xscale || !wq || !wscale || !out) return TG_ERR_INVALID_ARG;
  if (!aligned16(xq) || !aligned16(wq) || !aligned16(out)) return TG_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(xscale) & 3u) || (reinterpret_cast<uintptr_t>(wscale) & 3u))
    return TG_ERR_MISALIGNED;

  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;

  int bn, pair;
  pick_gemm_config(M, N, dev, info.sms, &bn, &pair);
  const int ch_bytes = (bn * esz) % 128 == 0 ? 128 : 64;  // epilogue chunk row bytes (kernel's CH_BYTES)

  CUtensorMap ta, tb, to;
  if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, uint64_t(K), uint64_t(M), uint64_t(K), BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return TG_ERR_CUDA;
  if (!make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, uint64_t(K), uint64_t(N), uint64_t(K), BK,
                    uint32_t(tg::gemm::b_rows(bn, pair != 0)), CU_TENSOR_MAP_SWIZZLE_128B))
    return TG_ERR_CUDA;
  const CUtensorMapDataType odt = out_dtype == TG_DT_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : out_dtype == TG_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!make_tmap_2d(&to, odt, out, uint64_t(N), uint64_t(M), uint64_t(N) * esz, uint32_t(ch_bytes / esz), 32,
                    ch_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
    return TG_ERR_CUDA;

  tg::GemmParams p;
  p.xscale = xscale;
  p.wscale = wscale;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.wscale_bcast = wscale_numel == 1 ? 1 : 0;
  p.M = int(M);
  p.N = int(N);
  p.K = int(K);
  p.m_tiles = int((M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM));
  p.n_tiles = int((N + bn - 1) / bn);
  p.k_blocks = int((K + int64_t(BK) * tg::gemm::ksub(pair != 0) - 1) / (int64_t(BK) * tg::gemm::ksub(pair != 0)));

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool hb = bias != nullptr;
  const int units = gemm_units(dev, info.sms, pair != 0);
  return pair ? launch_gemm_mode<true>(bn, ta, tb, to, p, out_dtype, hb, dev, units, st)
              : launch_gemm_mode<false>(bn, ta, tb, to, p, out_dtype, hb, dev, units, st);
}

int tg_set_sm_budget(int sms) {
  if (sms < 0) return TG_ERR_INVALID_ARG;
  g_sm_budget.store(sms, std::memory_order_relaxed);
  return TG_OK;
}

int tg_sm_budget(void) { return g_sm_budget.load(std::memory_order_relaxed); }

int tg_set_gemm_config(int bn, int pair) {
  if (pair < -1 || pair > 1) return TG_ERR_INVALID_ARG;
  bool ok = bn == 0;
  for (int w : kGemmWidths) ok = ok || w == bn;
  if (!ok) return TG_ERR_INVALID_ARG;
  g_forced_bn = bn;
  g_forced_pair = pair;
  return TG_OK;
}

int tg_gemm_config(int64_t M, int64_t N, int* bn, int* pair) {
  if (!bn || !pair) return TG_ERR_INVALID_ARG;
  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;
  pick_gemm_config(M, N, dev, info.sms, bn, pair);
  return TG_OK;
}

int tg_device_status(int device, uint32_t* bits, int clear) {
  if (!bits) return TG_ERR_INVALID_ARG;
  int prev;
  if (cudaGetDevice(&prev) != cudaSuccess) return TG_ERR_CUDA;
  if (device != prev && cudaSetDevice(device) != cudaSuccess) return TG_ERR_CUDA;
  unsigned int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, tg::g_device_status, sizeof(v));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(tg::g_device_status, &zero, sizeof(zero));
  }
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return TG_ERR_CUDA;
  *bits = v;
  return v ? TG_ERR_DEVICE_TIMEOUT : TG_OK;
}

}  // extern "C"

// ------------------------------------------------------------ small-M GEMM
namespace {

size_t round256(size_t v) { return (v + 255) & ~size_t(255); }

// The argument checks of tg_int8_gemm_dequant (M == 0 passes).
int check_gemm_args(const int8_t* xq, const float* xscale, const int8_t* wq, const float* wscale,
                    int64_t wscale_numel, const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K,
                    int out_dtype, const void* out) {
  if (M < 0 || N <= 0 || K <= 0) return TG_ERR_INVALID_ARG;
  if (out_dtype != TG_DT_F32 && out_dtype != TG_DT_F16 && out_dtype != TG_DT_BF16) return TG_ERR_INVALID_ARG;
  if (bias && bias_dtype != TG_DT_F32 && bias_dtype != TG_DT_F16 && bias_dtype != TG_DT_BF16)
    return TG_ERR_INVALID_ARG;
  if (wscale_numel != 1 && wscale_numel != N) return TG_ERR_INVALID_ARG;
  const int esz = out_dtype == TG_DT_F32 ? 4 : 2;
  if (K % 16 != 0 || (N * esz) % 16 != 0) return TG_ERR_UNSUPPORTED;
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31)) return TG_ERR_UNSUPPORTED;
  if (M == 0) return TG_OK;
  if (!xq || !xscale || !wq || !wscale || !out) return TG_ERR_INVALID_ARG;
  if (!aligned16(xq) || !aligned16(wq) || !aligned16(out)) return TG_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(xscale) & 3u) || (reinterpret_cast<uintptr_t>(wscale) & 3u))
    return TG_ERR_MISALIGNED;
  return TG_OK;
}

// Workspace of the split-K GEMM: [count: ceil(N/128) u32 | acc: M x N int32],
// each part 256-byte aligned.
struct SplitKWs {
  size_t count, acc, total;
};
SplitKWs splitk_ws(int64_t M, int64_t N) {
  SplitKWs w;
  const int64_t tiles = (N + tg::splitk::BNW - 1) / tg::splitk::BNW;
  w.count = 0;
  w.acc = round256(size_t(tiles) * 4);
  w.total = w.acc + round256(size_t(M) * size_t(N) * 4);
  return w;
}

// Whether the cluster form of the split-K kernel runs with `slices` CTAs per
// cluster on device `dev`: at most 8, and the occupancy calculator schedules at
// least one such cluster (cached per device and size).
template <int MPAD, int OUT, bool HAS_BIAS>
bool splitk_cluster_ok(int slices, int dev) {
  static uint32_t attr_done[kMaxDevices];
  static uint8_t ok_cache[kMaxDevices][9];  // 0 unknown, 1 yes, 2 no
  if (slices < 1 || slices > 8) return false;
  constexpr uint32_t smem = tg::splitk::smem_bytes(MPAD);
  auto kcl = tg::gemm_i8_splitk_kernel<MPAD, OUT, HAS_BIAS, true>;
  if (!ensure_smem_attr(kcl, dev, smem, attr_done)) {
    cudaGetLastError();
    return false;
  }
  uint8_t& ok = ok_cache[dev][slices];
  if (ok == 0) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(unsigned(slices), 1);
    cfg.blockDim = dim3(tg::splitk::THREADS);
    cfg.dynamicSmemBytes = smem;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(slices);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    ok = (cudaOccupancyMaxActiveClusters(&n, kcl, &cfg) == cudaSuccess && n > 0) ? 1 : 2;
    cudaGetLastError();  // a refusal here only selects the other form
  }
  return ok == 1;
}

template <int MPAD, int OUT, bool HAS_BIAS>
int launch_splitk_t(const CUtensorMap& tw, const CUtensorMap& tx, const tg::SplitKParams& p, int tiles, int dev,
                    cudaStream_t st) {
  static uint32_t attr_done[kMaxDevices];
  constexpr uint32_t smem = tg::splitk::smem_bytes(MPAD);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3(unsigned(p.slices), unsigned(tiles));
  cfg.blockDim = dim3(tg::splitk::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = unsigned(p.slices);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  // The slices of a column tile as one cluster, reduced in shared memory,
  // when K is split at most 8 ways and such a cluster fits on the device.
  if (splitk_cluster_ok<MPAD, OUT, HAS_BIAS>(p.slices, dev)) {
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, tg::gemm_i8_splitk_kernel<MPAD, OUT, HAS_BIAS, true>, tw, tx, p) != cudaSuccess)
      return TG_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? TG_OK : TG_ERR_CUDA;
  }
  auto kern = tg::gemm_i8_splitk_kernel<MPAD, OUT, HAS_BIAS, false>;
  if (!ensure_smem_attr(kern, dev, smem, attr_done)) return TG_ERR_CUDA;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, tw, tx, p) != cudaSuccess) return TG_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TG_OK : TG_ERR_CUDA;
}

template <int MPAD>
int launch_splitk_m(const CUtensorMap& tw, const CUtensorMap& tx, const tg::SplitKParams& p, int tiles,
                    int out_dtype, bool hb, int dev, cudaStream_t st) {
  switch (out_dtype) {
    case TG_DT_F32: return hb ? launch_splitk_t<MPAD, 0, true>(tw, tx, p, tiles, dev, st)
                              : launch_splitk_t<MPAD, 0, false>(tw, tx, p, tiles, dev, st);
    case TG_DT_F16: return hb ? launch_splitk_t<MPAD, 1, true>(tw, tx, p, tiles, dev, st)
                              : launch_splitk_t<MPAD, 1, false>(tw, tx, p, tiles, dev, st);
    default: return hb ? launch_splitk_t<MPAD, 2, true>(tw, tx, p, tiles, dev, st)
                       : launch_splitk_t<MPAD, 2, false>(tw, tx, p, tiles, dev, st);
  }
}

// K split of the small-M GEMM: about 1.6 CTAs per SM stream the weight
// (measured at M=1 on the DiT shapes: more in flight costs DRAM efficiency,
// fewer leaves bandwidth unused), so K is split until tiles x slices is nearest
// that, every slice non-empty.  Returns the slice count; *kb_per = k-blocks each.
int splitk_slices(int64_t N, int64_t K, int sms, int* kb_per) {
  using namespace tg::splitk;
  const int tiles = int((N + BNW - 1) / BNW);
  const int k_blocks = int((K + BK - 1) / BK);
  int slices = (16 * sms / 10 + tiles / 2) / tiles;
  slices = slices < 1 ? 1 : (slices > k_blocks ? k_blocks : slices);
  *kb_per = (k_blocks + slices - 1) / slices;
  return (k_blocks + *kb_per - 1) / *kb_per;
}

// The split-K launch over a zero-initialised scratch (count, acc), shared by
// the workspace entry point and any other caller that owns such scratch.
int splitk_launch(const int8_t* xq, const float* xscale, const int8_t* wq, const float* wscale,
                  int64_t wscale_numel, const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K,
                  int out_dtype, void* out, uint32_t* count, int32_t* acc, void* stream) {
  using namespace tg::splitk;
  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;
  const int mpad = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  const int tiles = int((N + BNW - 1) / BNW);
  const int k_blocks = int((K + BK - 1) / BK);
  int kb_per;
  const int slices = splitk_slices(N, K, info.sms, &kb_per);

  CUtensorMap tw, tx;
  if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, uint64_t(K), uint64_t(N), uint64_t(K), BK, BNW,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return TG_ERR_CUDA;
  if (!make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, uint64_t(K), uint64_t(M), uint64_t(K), BK,
                    uint32_t(mpad), CU_TENSOR_MAP_SWIZZLE_128B))
    return TG_ERR_CUDA;
  tg::SplitKParams p;
  p.xscale = xscale;
  p.wscale = wscale;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.wscale_bcast = wscale_numel == 1 ? 1 : 0;
  p.M = int(M);
  p.N = int(N);
  p.K = int(K);
  p.k_blocks = k_blocks;
  p.kb_per_slice = kb_per;
  p.slices = slices;
  p.acc = acc;
  p.count = count;
  p.out = out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool hb = bias != nullptr;
  switch (mpad) {
    case 16: return launch_splitk_m<16>(tw, tx, p, tiles, out_dtype, hb, dev, st);
    case 32: return launch_splitk_m<32>(tw, tx, p, tiles, out_dtype, hb, dev, st);
    case 64: return launch_splitk_m<64>(tw, tx, p, tiles, out_dtype, hb, dev, st);
    default: return launch_splitk_m<128>(tw, tx, p, tiles, out_dtype, hb, dev, st);
  }
}

}  // namespace

extern "C" {

size_t tg_int8_gemm_dequant_splitk_workspace(int64_t M, int64_t N) {
  if (M < 0 || N < 0) return 0;
  return splitk_ws(M, N).total;
}

int tg_int8_gemm_dequant_splitk(const int8_t* xq, const float* xscale, const int8_t* wq, const float* wscale,
                                int64_t wscale_numel, const void* bias, int bias_dtype, int64_t M, int64_t N,
                                int64_t K, int out_dtype, void* out, void* workspace, size_t workspace_bytes,
                                void* stream) {
  const int chk = check_gemm_args(xq, xscale, wq, wscale, wscale_numel, bias, bias_dtype, M, N, K, out_dtype, out);
  if (chk != TG_OK || M == 0) return chk;
  if (M > tg::splitk::M_MAX) return TG_ERR_UNSUPPORTED;
  if (!workspace) return TG_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return TG_ERR_MISALIGNED;
  const SplitKWs L = splitk_ws(M, N);
  if (workspace_bytes < L.total) return TG_ERR_INVALID_ARG;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  return splitk_launch(xq, xscale, wq, wscale, wscale_numel, bias, bias_dtype, M, N, K, out_dtype, out,
                       reinterpret_cast<uint32_t*>(ws + L.count), reinterpret_cast<int32_t*>(ws + L.acc), stream);
}

int64_t tg_int8_gemm_dequant_splitk_max_m(void) { return tg::splitk::M_MAX; }

int tg_int8_gemm_dequant_splitk_config(int64_t M, int64_t N, int64_t K, int out_dtype, int has_bias, int* slices,
                                       int* cluster) {
  if (M < 1 || M > tg::splitk::M_MAX || N < 1 || K < 1 || !slices || !cluster) return TG_ERR_INVALID_ARG;
  if (out_dtype != TG_DT_F32 && out_dtype != TG_DT_F16 && out_dtype != TG_DT_BF16) return TG_ERR_INVALID_ARG;
  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;
  int kb_per;
  const int s = splitk_slices(N, K, info.sms, &kb_per);
  const int mpad = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  const bool hb = has_bias != 0;
#define TG_SK_OK(MP, O) (hb ? splitk_cluster_ok<MP, O, true>(s, dev) : splitk_cluster_ok<MP, O, false>(s, dev))
#define TG_SK_OUT(MP) (out_dtype == TG_DT_F32 ? TG_SK_OK(MP, 0) : out_dtype == TG_DT_F16 ? TG_SK_OK(MP, 1) : TG_SK_OK(MP, 2))
  const bool cl = mpad == 16 ? TG_SK_OUT(16) : mpad == 32 ? TG_SK_OUT(32) : mpad == 64 ? TG_SK_OUT(64) : TG_SK_OUT(128);
#undef TG_SK_OUT
#undef TG_SK_OK
  *slices = s;
  *cluster = cl ? 1 : 0;
  return TG_OK;
}

}  // extern "C"

// ------------------------------------------------------------ few-row GEMV
namespace {

template <int MR, int OUT, bool HAS_BIAS>
int launch_gemv_t(const tg::GemvParams& p, int ctas, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(unsigned(ctas));
  cfg.blockDim = dim3(tg::gemv::THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, tg::gemv_i8_kernel<MR, OUT, HAS_BIAS>, p) != cudaSuccess) return TG_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TG_OK : TG_ERR_CUDA;
}

template <int MR>
int launch_gemv_m(const tg::GemvParams& p, int ctas, int out_dtype, bool hb, cudaStream_t st) {
  switch (out_dtype) {
    case TG_DT_F32: return hb ? launch_gemv_t<MR, 0, true>(p, ctas, st) : launch_gemv_t<MR, 0, false>(p, ctas, st);
    case TG_DT_F16: return hb ? launch_gemv_t<MR, 1, true>(p, ctas, st) : launch_gemv_t<MR, 1, false>(p, ctas, st);
    default: return hb ? launch_gemv_t<MR, 2, true>(p, ctas, st) : launch_gemv_t<MR, 2, false>(p, ctas, st);
  }
}

// K parts per group of 4 weight rows: the fewest of 1, 2, 4, 8 that put at
// least two CTAs (16 warps) per SM on the weight stream, each part keeping
// at least one 16-byte chunk per lane.
int gemv_parts(int64_t N, int64_t K, int sms) {
  using namespace tg::gemv;
  const int64_t groups = N / R;
  const int64_t nch = K / 16;
  int kp = 1;
  while (kp < WARPS && (groups * kp + WARPS - 1) / WARPS < 2 * int64_t(sms) && nch >= int64_t(64) * kp) kp *= 2;
  return kp;
}

// Weights up to this size have a quarter asked into L2 before the wait (the
// L2 holds 126 MB, so the quarter stays there until it is read); larger ones
// stream without the prefetch.
constexpr int64_t kGemvPrefetchMaxBytes = int64_t(256) << 20;

}  // namespace

extern "C" {

int tg_int8_gemv_dequant(const int8_t* xq, const float* xscale, const int8_t* wq, const float* wscale,
                         int64_t wscale_numel, const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K,
                         int out_dtype, void* out, void* stream) {
  const int chk = check_gemm_args(xq, xscale, wq, wscale, wscale_numel, bias, bias_dtype, M, N, K, out_dtype, out);
  if (chk != TG_OK || M == 0) return chk;
  if (M > TG_GEMV_MAX_M) return TG_ERR_UNSUPPORTED;
  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;
  using namespace tg::gemv;
  const int kp = gemv_parts(N, K, info.sms_all);
  const int64_t nch = K / 16;
  const int64_t groups = N / R;  // N is a multiple of 4 (16-byte output rows)
  const int64_t per_cta = WARPS / kp;
  const int64_t ctas = (groups + per_cta - 1) / per_cta;
  if (ctas > 0x7fffffff) return TG_ERR_UNSUPPORTED;
  tg::GemvParams p;
  p.xq = xq;
  p.xscale = xscale;
  p.wq = wq;
  p.wscale = wscale;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.wscale_bcast = wscale_numel == 1 ? 1 : 0;
  p.M = int(M);
  p.N = int(N);
  p.K = int(K);
  p.kp = kp;
  p.part_chunks = int((nch + kp - 1) / kp);
  p.prefetch = N * K <= kGemvPrefetchMaxBytes ? 1 : 0;
  p.out = out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool hb = bias != nullptr;
  switch (M) {
    case 1: return launch_gemv_m<1>(p, int(ctas), out_dtype, hb, st);
    case 2: return launch_gemv_m<2>(p, int(ctas), out_dtype, hb, st);
    default: return launch_gemv_m<4>(p, int(ctas), out_dtype, hb, st);
  }
}

int tg_int8_gemv_dequant_config(int64_t N, int64_t K, int* parts, int* ctas) {
  if (N < 1 || K < 16 || !parts || !ctas) return TG_ERR_INVALID_ARG;
  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;
  const int kp = gemv_parts(N, K, info.sms_all);
  const int64_t per_cta = tg::gemv::WARPS / kp;
  *parts = kp;
  *ctas = int((N / tg::gemv::R + per_cta - 1) / per_cta);
  return TG_OK;
}

}  // extern "C"

// ------------------------------------------------------------ no-allocation variant
// The split-K GEMM for callers that must not allocate device memory.  Its
// scratch is this file-scope array, sized for at most 2^20 accumulator
// elements (M x N, 4 MiB) and N <= 65536 (2 KiB of tile counters): 4 MiB + 2 KiB
// that every GPU which loads the library keeps until the process exits.
namespace {

constexpr int64_t kNoAllocMaxM = 64;
constexpr int64_t kNoAllocMaxN = 65536;
constexpr int64_t kNoAllocMaxAcc = int64_t(1) << 20;
constexpr size_t kNoAllocCountBytes = size_t(kNoAllocMaxN / tg::splitk::BNW) * 4;  // 256-byte multiple
constexpr size_t kNoAllocBytes = kNoAllocCountBytes + size_t(kNoAllocMaxAcc) * 4;

static __device__ __align__(256) unsigned char g_splitk_scratch[kNoAllocBytes];

// Device address of g_splitk_scratch on `dev` (the current device).  In host
// code the array's name only stands in for the symbol; its address on a
// device comes from the runtime, once per device.
bool noalloc_scratch(int dev, uint8_t** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices];
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_splitk_scratch) != cudaSuccess || p == nullptr) return false;
    addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(addr[dev]);
  return true;
}

}  // namespace

extern "C" {

int tg_int8_gemm_dequant_splitk_noalloc(const int8_t* xq, const float* xscale, const int8_t* wq,
                                        const float* wscale, int64_t wscale_numel, const void* bias, int bias_dtype,
                                        int64_t M, int64_t N, int64_t K, int out_dtype, void* out, void* stream) {
  const int chk = check_gemm_args(xq, xscale, wq, wscale, wscale_numel, bias, bias_dtype, M, N, K, out_dtype, out);
  if (chk != TG_OK || M == 0) return chk;
  if (M > kNoAllocMaxM || N > kNoAllocMaxN || M * N > kNoAllocMaxAcc) return TG_ERR_UNSUPPORTED;
  int dev;
  DeviceInfo info;
  if (!current_device(&dev, &info)) return TG_ERR_CUDA;
  uint8_t* scratch = nullptr;
  if (!noalloc_scratch(dev, &scratch)) return TG_ERR_CUDA;
  // Every call shares the array: when the sums go through it (K split more
  // than a cluster holds), zero the counters and this call's part of the
  // accumulator first, in stream order (a memset, not an allocation).  The
  // cluster form sums in shared memory and never touches the array.
  int slices = 0, cluster = 0;
  const int cfg = tg_int8_gemm_dequant_splitk_config(M, N, K, out_dtype, bias != nullptr, &slices, &cluster);
  if (cfg != TG_OK) return cfg;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!cluster && cudaMemsetAsync(scratch, 0, kNoAllocCountBytes + size_t(M) * size_t(N) * 4, st) != cudaSuccess)
    return TG_ERR_CUDA;
  return splitk_launch(xq, xscale, wq, wscale, wscale_numel, bias, bias_dtype, M, N, K, out_dtype, out,
                       reinterpret_cast<uint32_t*>(scratch), reinterpret_cast<int32_t*>(scratch + kNoAllocCountBytes),
                       stream);
}

}  // extern "C"

// ------------------------------------------------------------------ peer memory
// Buffers that other processes on this node (one per GPU) can map, and copies
// between mapped buffers on a stream.  cudaMemcpyAsync between this device and
// a peer's mapped memory runs on a copy engine over NVLink, using no SMs.
extern "C" {

size_t tg_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int tg_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return TG_ERR_INVALID_ARG;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return TG_ERR_CUDA;
  if (cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p) != cudaSuccess) {
    cudaFree(p);
    return TG_ERR_CUDA;
  }
  *ptr = p;
  return TG_OK;
}

int tg_peer_free(void* ptr) {
  if (!ptr) return TG_ERR_INVALID_ARG;
  return cudaFree(ptr) == cudaSuccess ? TG_OK : TG_ERR_CUDA;
}

int tg_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return TG_ERR_INVALID_ARG;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return TG_ERR_CUDA;
  *ptr = p;
  return TG_OK;
}

int tg_peer_close(void* ptr) {
  if (!ptr) return TG_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? TG_OK : TG_ERR_CUDA;
}

int tg_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return TG_OK;
  if (!dst || !src) return TG_ERR_INVALID_ARG;
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? TG_OK
             : TG_ERR_CUDA;
}

}  // extern "C"
