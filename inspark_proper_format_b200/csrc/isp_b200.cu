// C-ABI entry points of libisp_b200.so (single translation unit: every kernel
// header is included here so the device error word is shared).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "conv.cuh"
#include "fir.cuh"
#include "gemm_sm100.cuh"
#include "decode_sm100.cuh"
#include "norm_quant.cuh"

namespace isp {

int check_device() {
  static std::mutex mu;
  static int cached[64];
  static bool init = false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ISP_ERR_ARCH;
  std::lock_guard<std::mutex> lock(mu);
  if (!init) {
    for (int& c : cached) c = -1;
    init = true;
  }
  if (dev < 0 || dev >= 64) return ISP_ERR_ARCH;
  if (cached[dev] < 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cached[dev] = (major == 10 && minor == 0) ? ISP_OK : ISP_ERR_ARCH;
  }
  return cached[dev];
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

namespace gemm {

using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// 2-D row-major tensor [outer, inner] with a (box_inner x box_outer) box and 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
              uint64_t outer, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D row-major uint8 tensor [d2, d1, d0] (d0 innermost) with a (box0 x box1 x 1) box, 128-byte swizzle.
bool make_map3d_u8(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t box0,
                   uint32_t box1) {
  EncodeFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0, d0 * d1};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [B, CO, T_out] convolution output: boxes of 32/P channels x 32P times (one epilogue
// warp's 32 phase rows x 32 folded columns), no swizzle.
bool make_conv_out_map(CUtensorMap* map, void* y, int out_kind, uint64_t t_out, uint64_t co, uint64_t b,
                       uint32_t phases) {
  EncodeFn fn = encode_fn();
  if (fn == nullptr) return false;
  const int eb = out_bytes(out_kind);
  const CUtensorMapDataType dt = out_kind == OUT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : out_kind == OUT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {t_out, co, b};
  cuuint64_t strides[2] = {t_out * eb, t_out * eb * co};
  cuuint32_t box[3] = {32u * phases, 32u / phases, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(map, dt, 3, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_out_map(CUtensorMap* map, void* out, int out_kind, int64_t M, int N) {
  const int eb = out_bytes(out_kind);
  const CUtensorMapDataType dt = out_kind == OUT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : out_kind == OUT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : out_kind == OUT_F16  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  return make_map(map, out, dt, eb, static_cast<uint64_t>(N), static_cast<uint64_t>(M),
                  static_cast<uint32_t>(128 / eb), 32);
}


#ifndef ISP_GEMM_STAGES
#define ISP_GEMM_STAGES 4
#endif
#ifndef ISP_GEMM_SCALE_EPI_WARPS
#define ISP_GEMM_SCALE_EPI_WARPS 8
#endif
constexpr int kBN = 256;
constexpr int kStages = ISP_GEMM_STAGES;
constexpr int kScaleEpiWarps = ISP_GEMM_SCALE_EPI_WARPS;   // scale/bias/residual epilogues
constexpr int kSwigluEpiWarps = 4;                         // SwiGLU: 128 output columns per tile

// NVFP4: 128 x 128 tiles (two 128-column accumulators + 32 scale columns per
// stage in TMEM); a stage is 16 KB of A, 16 KB of B and 4 KB of scales.
#ifndef ISP_GEMM_FP4_STAGES
#define ISP_GEMM_FP4_STAGES 5
#endif
constexpr int kFp4BN = 128;
constexpr int kFp4Stages = ISP_GEMM_FP4_STAGES;
constexpr int kFp4SwigluEpiWarps = 16;   // one NVFP4 block (16 outputs) per thread per tile

// B-stationary schedule (K bytes <= kStatK): the whole B tile stays in shared
// memory and only A streams, a third of the operand traffic of a 128 x 256 FP8
// tile (the streaming schedule is bound by L2 -> SM bandwidth).
constexpr int kStatK = 512;
constexpr int kStatStages = 4;         // FP8 / INT8: 4 x 16 KB of A + 128 KB of B
constexpr int kFp4StatStages = 6;      // NVFP4: 6 x 18 KB of A (+ scales) + 72 KB of B (+ scales)
constexpr int kNlvStatStages = 6;      // INT8 nonlinear value: 6 x 16 KB of A + 96 KB of B (3 x 64 rows)
// SM pairs: each CTA holds half of the B tile (64 KB at K = 512), which leaves room for
// six 16 KB A stages and two staging boxes per epilogue warp.
#ifndef ISP_GEMM_PAIR_STAGES
#define ISP_GEMM_PAIR_STAGES 6
#endif
constexpr int kPairStages = ISP_GEMM_PAIR_STAGES;
// Streaming SM pairs (K > 512 bytes): a stage is 16 KB of A and 16 KB of B (this CTA's
// half of the 256 B rows); five stages beside two staging boxes per epilogue warp.
constexpr int kPairStreamStages = 5;

// Schedule overrides for A/B measurements, fixed at compile time (e.g.
// -DISP_GEMM_FORCE_STREAMING=1); the shipped library defines none of them, so it
// has one code path per shape and no run-time switch.
//   ISP_GEMM_FORCE_STREAMING  stream B through the ring even when K fits the resident tile
//   ISP_GEMM_NO_TAIL_SPLIT    keep the last partial wave of streaming GEMMs as whole tiles
//   ISP_CONV_DIRECT_STORE     per-element stores in the convolution epilogue
//   ISP_GEMM_NO_DECODE        the regular kernel for M <= 128 instead of cluster split-K
//   ISP_GEMM_NO_PAIR          scale GEMMs on one CTA per tile instead of SM pairs
#ifndef ISP_GEMM_FORCE_STREAMING
#define ISP_GEMM_FORCE_STREAMING 0
#endif
#ifndef ISP_GEMM_NO_TAIL_SPLIT
#define ISP_GEMM_NO_TAIL_SPLIT 0
#endif
#ifndef ISP_CONV_DIRECT_STORE
#define ISP_CONV_DIRECT_STORE 0
#endif
#ifndef ISP_GEMM_NO_DECODE
#define ISP_GEMM_NO_DECODE 0
#endif
#ifndef ISP_GEMM_NO_PAIR
#define ISP_GEMM_NO_PAIR 0
#endif
constexpr bool streaming_forced() { return ISP_GEMM_FORCE_STREAMING != 0; }
constexpr bool tail_split_disabled() { return ISP_GEMM_NO_TAIL_SPLIT != 0; }
constexpr bool conv_direct_forced() { return ISP_CONV_DIRECT_STORE != 0; }
constexpr bool decode_disabled() { return ISP_GEMM_NO_DECODE != 0; }
constexpr bool pair_schedule_enabled() { return ISP_GEMM_NO_PAIR == 0; }

template <int kBN, int kStages, int kEpiWarps, int kAB, int kEpi, int kOut, int kBStatK = 0, bool kPair = false>
int launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& b2, const CUtensorMap& o,
           const Params& p, cudaStream_t stream) {
  auto kern = gemm_kernel<kBN, kStages, kEpiWarps, kAB, kEpi, kOut, kBStatK, kPair>;
  constexpr int kSmem = Smem<kPair ? kBN / 2 : kBN, kStages, kEpiWarps, kAB == AB_FP4, kOut != OUT_NVFP4 && kEpi != EPI_NLV,
                             kBStatK, kPair ? kStagingBufsPair : kStagingBufsOne>::kBytes;
  static_assert(kSmem <= 232448, "shared memory budget of one sm_100 CTA");
  static bool configured[64] = {false};
  static int max_pairs[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return ISP_ERR_LAUNCH;
    if constexpr (kPair) {
      // persistent pairs: no more clusters than can be resident at once
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (sm_count() / 2));
      cfg.blockDim = dim3(kernel_threads<kEpiWarps, kAB == AB_FP4>());
      cfg.dynamicSmemBytes = kSmem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = sm_count() / 2;
      }
      max_pairs[dev] = n < sm_count() / 2 ? n : sm_count() / 2;
    }
    configured[dev] = true;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  if constexpr (kPair) {
    const int cap = (dev >= 0 && dev < 64 && max_pairs[dev] > 0) ? max_pairs[dev] : sm_count() / 2;
    const int pairs = tiles < cap ? tiles : cap;
    return launch_pdl_cluster(kern, dim3(2 * pairs), dim3(kernel_threads<kEpiWarps, kAB == AB_FP4>()), kSmem, stream, 2u, a, b, b2,
                              o, p);
  }
  const int grid = tiles < sm_count() ? tiles : sm_count();
  return launch_pdl(kern, dim3(grid), dim3(kernel_threads<kEpiWarps, kAB == AB_FP4>()), kSmem, stream, a, b, b2, o, p);
}

// Schedules: 0 streaming, 1 B-stationary (one CTA per tile), 2 B-stationary SM pairs.
enum Sched { SCHED_STREAM = 0, SCHED_STAT = 1, SCHED_PAIR = 2, SCHED_PAIR_STREAM = 3 };
constexpr bool sched_pair(int s) { return s == SCHED_PAIR || s == SCHED_PAIR_STREAM; }

template <int kAB, int kOut>
int launch_scale(int sched, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o, const Params& p,
                 cudaStream_t s) {
  if constexpr (kAB == AB_FP4) {
    return sched != SCHED_STREAM
               ? launch<kFp4BN, kFp4StatStages, kScaleEpiWarps, kAB, EPI_SCALE, kOut, kStatK>(a, b, b, o, p, s)
               : launch<kFp4BN, kFp4Stages, kScaleEpiWarps, kAB, EPI_SCALE, kOut>(a, b, b, o, p, s);
  } else {
    if (sched == SCHED_PAIR)
      return launch<kBN, kPairStages, kScaleEpiWarps, kAB, EPI_SCALE, kOut, kStatK, true>(a, b, b, o, p, s);
    if (sched == SCHED_PAIR_STREAM)
      return launch<kBN, kPairStreamStages, kScaleEpiWarps, kAB, EPI_SCALE, kOut, 0, true>(a, b, b, o, p, s);
    return sched == SCHED_STAT ? launch<kBN, kStatStages, kScaleEpiWarps, kAB, EPI_SCALE, kOut, kStatK>(a, b, b, o, p, s)
                               : launch<kBN, kStages, kScaleEpiWarps, kAB, EPI_SCALE, kOut>(a, b, b, o, p, s);
  }
}

template <int kAB>
int dispatch_scale_out(int out_kind, int sched, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o,
                       const Params& p, cudaStream_t s) {
  switch (out_kind) {
    case OUT_BF16: return launch_scale<kAB, OUT_BF16>(sched, a, b, o, p, s);
    case OUT_F16: return launch_scale<kAB, OUT_F16>(sched, a, b, o, p, s);
    case OUT_F32: return launch_scale<kAB, OUT_F32>(sched, a, b, o, p, s);
    case OUT_E4M3:
      if constexpr (kAB == AB_FP4) return ISP_ERR_DTYPE;
      else return launch_scale<kAB, OUT_E4M3>(sched, a, b, o, p, s);
    default: return ISP_ERR_DTYPE;
  }
}

bool global_scale_ok(float g) { return g >= 0x1p-100f && g <= 0x1p100f; }

// Row-major E4M3 scales [R, K/16] -> tensor-core layout; one thread per
// 4-byte word (the 4 scales of one row in one 64-element K chunk).
__global__ void scales_to_mma_kernel(const uint32_t* src, int64_t R, int kchunks, uint32_t* dst, int64_t words) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w >= words) return;
  const int64_t r = w / kchunks;
  const int c = static_cast<int>(w - r * kchunks);
  const uint32_t v = r < R ? __ldg(src + r * kchunks + c) : 0u;
  const int64_t off = ((r >> 7) * kchunks + c) * 128 + (r & 31) * 4 + ((r >> 5) & 3);   // in words
  dst[off] = v;
}

// Small-M path: cluster split-K (decode_sm100.cuh).
template <bool kInt8, int kOut>
int launch_decode(const CUtensorMap& a, const CUtensorMap& b, const Params& p, int splits, int n_tiles,
                  cudaStream_t stream) {
  auto kern = decode_kernel<kInt8, kOut>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DecSmem::kBytes) != cudaSuccess)
      return ISP_ERR_LAUNCH;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(n_tiles), 1);
  cfg.blockDim = dim3(kDecThreads, 1, 1);
  cfg.dynamicSmemBytes = DecSmem::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see pdl_wait()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, a, b, p, splits) != cudaSuccess) {
    cudaGetLastError();
    return ISP_ERR_LAUNCH;
  }
  return launch_status();
}

template <bool kInt8>
int dispatch_decode(int out_kind, const CUtensorMap& a, const CUtensorMap& b, const Params& p, int splits,
                    int n_tiles, cudaStream_t s) {
  switch (out_kind) {
    case OUT_BF16: return launch_decode<kInt8, OUT_BF16>(a, b, p, splits, n_tiles, s);
    case OUT_F16: return launch_decode<kInt8, OUT_F16>(a, b, p, splits, n_tiles, s);
    case OUT_F32: return launch_decode<kInt8, OUT_F32>(a, b, p, splits, n_tiles, s);
    default: return ISP_ERR_DTYPE;
  }
}

// Phase-folded form of a convolution: output time t = q * P + r is row q, column
// co * P + r of one GEMM whose K runs over window slots j (128-channel blocks each).
// Conv1d (stride S): P = 1, slot j is tap j at input position t * S + o,
// o = j * dilation - padding, which in the A view [rows / S, S * C_pad] is row
// t + floor(o / S), column block (o mod S) * C_pad / 128.
// ConvTranspose1d (stride S): P = S; output q * S + r gathers input q + R from tap k
// when r + padding - k * dilation = R * S; slot j covers R = r_min + j for every phase
// at once (taps that do not reach a (phase, slot) pair are zero weights).
struct ConvGeom {
  int phases, taps, a_stride, r_min;
  int row[kConvTab];
  int colstep[kConvTab];
};

inline int64_t floor_div(int64_t a, int64_t b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

int conv_geometry(int KW, int stride, int dilation, int padding, int transposed, ConvGeom* g) {
  // |row offsets| < 2^19 keeps row * 1024 + column in an int
  if (KW < 1 || stride < 1 || dilation < 1 || padding < 0 || KW > 4096 || stride > 4096 ||
      static_cast<int64_t>(dilation) * (KW - 1) + padding >= (1 << 19))
    return ISP_ERR_SHAPE;
  if (!transposed) {
    if (KW > kConvTab) return ISP_ERR_SHAPE;
    g->phases = 1;
    g->taps = KW;
    g->a_stride = stride;
    g->r_min = 0;
    for (int j = 0; j < KW; ++j) {
      const int64_t o = static_cast<int64_t>(j) * dilation - padding;
      const int64_t row = floor_div(o, stride);
      g->row[j] = static_cast<int>(row);
      g->colstep[j] = static_cast<int>(o - row * stride);
    }
    return ISP_OK;
  }
  int64_t lo = 0, hi = -1;
  for (int r = 0; r < stride; ++r)
    for (int k = 0; k < KW; ++k) {
      const int64_t num = static_cast<int64_t>(r) + padding - static_cast<int64_t>(k) * dilation;
      if (num % stride != 0) continue;
      const int64_t R = num / stride;
      if (hi < lo) lo = hi = R;
      lo = R < lo ? R : lo;
      hi = R > hi ? R : hi;
    }
  if (hi < lo) lo = hi = 0;                    // no tap reaches any output: one zero slot
  if (hi - lo + 1 > kConvTab) return ISP_ERR_SHAPE;
  g->phases = stride;
  g->taps = static_cast<int>(hi - lo + 1);
  g->a_stride = 1;
  g->r_min = static_cast<int>(lo);
  for (int j = 0; j < g->taps; ++j) {
    g->row[j] = static_cast<int>(lo) + j;
    g->colstep[j] = 0;
  }
  return ISP_OK;
}

template <int kAB, int kOut>
int launch_conv(bool stat, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o, const Params& p,
                cudaStream_t s) {
  return stat ? launch<kBN, kStatStages, kScaleEpiWarps, kAB, EPI_CONV, kOut, kStatK>(a, b, b, o, p, s)
              : launch<kBN, kStages, kScaleEpiWarps, kAB, EPI_CONV, kOut>(a, b, b, o, p, s);
}

int out_kind_of(int dtype) {
  switch (dtype) {
    case ISP_BF16: return OUT_BF16;
    case ISP_F16: return OUT_F16;
    case ISP_F32: return OUT_F32;
    case ISP_E4M3: return OUT_E4M3;
    default: return -1;
  }
}

}  // namespace gemm
}  // namespace isp

// Per-utterance |x| maxima of isp_conv1d_dynamic_noalloc, kept in the library instead
// of a caller buffer.  One region per process and device: calls that overlap in time
// (two streams, two host threads) race on it.
constexpr int64_t kConvNoAllocMaxBatch = 8192;
static __device__ __align__(256) float g_conv_amax_scratch[kConvNoAllocMaxBatch];

extern "C" {

int isp_version(void) { return 100; }

const char* isp_status_string(int status) {
  switch (status) {
    case ISP_OK: return "ok";
    case ISP_ERR_SHAPE: return "unsupported shape";
    case ISP_ERR_ALIGN: return "pointer or row stride not 16-byte aligned";
    case ISP_ERR_DTYPE: return "unsupported dtype";
    case ISP_ERR_ARCH: return "current device is not an sm_100 (B200) GPU";
    case ISP_ERR_LAUNCH: return "CUDA launch failed";
    case ISP_ERR_TIMEOUT: return "a bounded device-side wait expired";
    case ISP_ERR_ARG: return "invalid argument";
    default: return "unknown status";
  }
}

int isp_device_check(void) { return isp::check_device(); }

int isp_read_device_error(int* error_out, int clear, isp_stream_t stream) {
  if (error_out == nullptr) return ISP_ERR_ARG;
  if (int st = isp::check_device()) return st;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return ISP_ERR_LAUNCH;
  int value = 0;
  if (cudaMemcpyFromSymbol(&value, isp::g_device_error, sizeof(int)) != cudaSuccess) return ISP_ERR_LAUNCH;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(isp::g_device_error, &zero, sizeof(int)) != cudaSuccess) return ISP_ERR_LAUNCH;
  }
  *error_out = value;
  return ISP_OK;
}

int isp_wait_selftest(int64_t limit_ns, isp_stream_t stream) {
  if (limit_ns < 1000 || limit_ns > 100000000) return ISP_ERR_ARG;    // 1 us .. 100 ms
  if (int st = isp::check_device()) return st;
  isp::gemm::wait_selftest_kernel<<<1, 96, 0, stream>>>(static_cast<uint64_t>(limit_ns));
  return isp::launch_status();
}

int isp_norm_quant(const void* x, int x_dtype, int64_t M, int K, const float* gamma,
                   const float* bias, float eps, float out_mul, int norm_kind, int qfmt,
                   float scale, const float* smooth, void* codes, void* scales_out,
                   isp_stream_t stream) {
  if (x == nullptr || codes == nullptr) return ISP_ERR_ARG;
  if (x_dtype != ISP_BF16 && x_dtype != ISP_F32) return ISP_ERR_DTYPE;
  if (M < 0 || K <= 0 || K % 16 != 0) return ISP_ERR_SHAPE;
  if (norm_kind < ISP_NORM_NONE || norm_kind > ISP_NORM_BIAS) return ISP_ERR_ARG;
  if (qfmt < ISP_Q_E4M3_STATIC || qfmt > ISP_Q_NVFP4_MMA) return ISP_ERR_ARG;
  const bool nvfp4 = qfmt == ISP_Q_NVFP4 || qfmt == ISP_Q_NVFP4_MMA;
  if (qfmt == ISP_Q_NVFP4_MMA && K % 64 != 0) return ISP_ERR_SHAPE;
  if ((norm_kind == ISP_NORM_RMS_GPTFAST || norm_kind == ISP_NORM_RMS_QWEN) && gamma == nullptr)
    return ISP_ERR_ARG;
  if (norm_kind == ISP_NORM_BIAS && bias == nullptr) return ISP_ERR_ARG;
  if ((qfmt == ISP_Q_E4M3_ROW || nvfp4) && scales_out == nullptr) return ISP_ERR_ARG;
  if (qfmt != ISP_Q_E4M3_ROW && !isp::gemm::global_scale_ok(scale)) return ISP_ERR_ARG;
  if (!isp::aligned16(x) || !isp::aligned16(codes)) return ISP_ERR_ALIGN;
  if ((gamma && !isp::aligned16(gamma)) || (bias && !isp::aligned16(bias)) ||
      (smooth && !isp::aligned16(smooth)))
    return ISP_ERR_ALIGN;
  if (qfmt == ISP_Q_NVFP4 && (reinterpret_cast<uintptr_t>(scales_out) & 1)) return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (M == 0) return ISP_OK;
  isp::NormQuantParams p{x, M, K, gamma, bias, eps, out_mul, scale, smooth, codes, scales_out, nullptr, nullptr, 1};
  return x_dtype == ISP_BF16 ? isp::launch_norm_quant_kind<true>(norm_kind, qfmt, p, stream)
                             : isp::launch_norm_quant_kind<false>(norm_kind, qfmt, p, stream);
}

int isp_adaln_quant(const void* x, int x_dtype, int64_t M, int K, const float* gamma, float eps, const float* ada_w,
                    const float* ada_b, int64_t rows_per_group, int qfmt, float scale, const float* smooth,
                    void* codes, void* scales_out, isp_stream_t stream) {
  if (ada_w == nullptr || ada_b == nullptr || gamma == nullptr) return ISP_ERR_ARG;
  if (rows_per_group <= 0 || M % rows_per_group != 0) return ISP_ERR_SHAPE;
  if (!isp::aligned16(ada_w) || !isp::aligned16(ada_b)) return ISP_ERR_ALIGN;
  // shared validation of the plain entry (norm kind fixed to gpt_fast RMSNorm)
  if (x == nullptr || codes == nullptr) return ISP_ERR_ARG;
  if (x_dtype != ISP_BF16 && x_dtype != ISP_F32) return ISP_ERR_DTYPE;
  if (M < 0 || K <= 0 || K % 16 != 0) return ISP_ERR_SHAPE;
  if (qfmt < ISP_Q_E4M3_STATIC || qfmt > ISP_Q_NVFP4_MMA) return ISP_ERR_ARG;
  const bool nvfp4 = qfmt == ISP_Q_NVFP4 || qfmt == ISP_Q_NVFP4_MMA;
  if (qfmt == ISP_Q_NVFP4_MMA && K % 64 != 0) return ISP_ERR_SHAPE;
  if ((qfmt == ISP_Q_E4M3_ROW || nvfp4) && scales_out == nullptr) return ISP_ERR_ARG;
  if (qfmt != ISP_Q_E4M3_ROW && !isp::gemm::global_scale_ok(scale)) return ISP_ERR_ARG;
  if (!isp::aligned16(x) || !isp::aligned16(codes) || !isp::aligned16(gamma) || (smooth && !isp::aligned16(smooth)))
    return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (M == 0) return ISP_OK;
  isp::NormQuantParams p{x, M, K, gamma, nullptr, eps, 1.f, scale, smooth, codes, scales_out, ada_w, ada_b,
                         rows_per_group};
  return x_dtype == ISP_BF16 ? isp::launch_norm_quant_kind<true>(ISP_NORM_RMS_GPTFAST, qfmt, p, stream)
                             : isp::launch_norm_quant_kind<false>(ISP_NORM_RMS_GPTFAST, qfmt, p, stream);
}

int isp_conv1d_geometry(int KW, int stride, int dilation, int padding, int transposed, int* phases, int* taps) {
  isp::gemm::ConvGeom g;
  if (phases == nullptr || taps == nullptr) return ISP_ERR_ARG;
  if (int st = isp::gemm::conv_geometry(KW, stride, dilation, padding, transposed, &g)) return st;
  *phases = g.phases;
  *taps = g.taps;
  return ISP_OK;
}

int isp_conv1d_pack_weight(const void* codes, int64_t ldw, int CO, int CI, int KW, int stride, int dilation,
                           int padding, int transposed, void* w_packed, int C_pad, isp_stream_t stream) {
  isp::gemm::ConvGeom g;
  if (codes == nullptr || w_packed == nullptr) return ISP_ERR_ARG;
  if (CO <= 0 || CI <= 0 || ldw < CO || C_pad < CI || C_pad % 128 != 0) return ISP_ERR_SHAPE;
  if (int st = isp::gemm::conv_geometry(KW, stride, dilation, padding, transposed, &g)) return st;
  if (!isp::aligned16(w_packed)) return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  isp::ConvPackParams p{};
  p.src = static_cast<const uint8_t*>(codes);
  p.ldw = ldw;
  p.CO = CO;
  p.CI = CI;
  p.KW = KW;
  p.phases = g.phases;
  p.taps = g.taps;
  p.c_pad = C_pad;
  p.transposed = transposed ? 1 : 0;
  p.stride = stride;
  p.dilation = dilation;
  p.padding = padding;
  p.r_min = g.r_min;
  p.dst = static_cast<uint8_t*>(w_packed);
  const int64_t total = static_cast<int64_t>(CO) * g.phases * g.taps * (C_pad / 16);
  isp::conv_pack_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(p);
  return isp::launch_status();
}

int isp_conv1d_quant(const void* x, int x_dtype, int64_t B, int C, int64_t T, int row_multiple, const float* smooth,
                     float in_scale, float* amax, int code_dtype, void* xq, int C_pad, isp_stream_t stream) {
  if (x == nullptr || xq == nullptr) return ISP_ERR_ARG;
  if (x_dtype != ISP_F32 && x_dtype != ISP_BF16) return ISP_ERR_DTYPE;
  if (code_dtype != ISP_E4M3 && code_dtype != ISP_I8) return ISP_ERR_DTYPE;
  if (smooth != nullptr && code_dtype != ISP_I8) return ISP_ERR_ARG;
  if (amax != nullptr && (code_dtype != ISP_E4M3 || in_scale != 0.f)) return ISP_ERR_ARG;
  if (amax == nullptr && !isp::gemm::global_scale_ok(in_scale)) return ISP_ERR_ARG;
  if (B < 0 || B > 65535 || C <= 0 || T <= 0 || row_multiple < 1 || C_pad < C || C_pad % 128 != 0)
    return ISP_ERR_SHAPE;
  if (!isp::aligned16(xq)) return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (B == 0) return ISP_OK;
  if (amax != nullptr) {
    if (cudaMemsetAsync(amax, 0, static_cast<size_t>(B) * sizeof(float), stream) != cudaSuccess)
      return ISP_ERR_LAUNCH;
    const int64_t per = static_cast<int64_t>(C) * T;
    const int64_t want = (per + 256 * 32 - 1) / (256 * 32);         // >= 32 elements per thread
    const int64_t cap = (4 * isp::sm_count() + B - 1) / B;     // ~4 blocks per SM over all utterances
    const unsigned bx = static_cast<unsigned>(want < cap ? (want > 0 ? want : 1) : cap);
    const dim3 grid(bx, static_cast<unsigned>(B));
    if (x_dtype == ISP_BF16) isp::conv_amax_kernel<true><<<grid, 256, 0, stream>>>(x, per, amax);
    else isp::conv_amax_kernel<false><<<grid, 256, 0, stream>>>(x, per, amax);
  }
  isp::ConvQuantParams p{};
  p.x = x;
  p.B = B;
  p.C = C;
  p.T = T;
  p.t_rows = (T + row_multiple - 1) / row_multiple * row_multiple;
  p.c_pad = C_pad;
  // RN(1/s): the host division is IEEE single precision, the reciprocal the kernels expect
  p.scale = amax != nullptr ? 1.f : in_scale;
  p.rscale = 1.f / p.scale;
  p.amax = amax;
  p.smooth = smooth;
  p.xq = static_cast<uint8_t*>(xq);
  const dim3 grid(static_cast<unsigned>((p.t_rows + isp::kCqRows - 1) / isp::kCqRows), static_cast<unsigned>(C_pad / 128),
                  static_cast<unsigned>(B));
  const bool bf16 = x_dtype == ISP_BF16;
  if (code_dtype == ISP_I8) {
    if (bf16) isp::conv_quant_kernel<true, true><<<grid, 256, 0, stream>>>(p);
    else isp::conv_quant_kernel<true, false><<<grid, 256, 0, stream>>>(p);
  } else {
    if (bf16) isp::conv_quant_kernel<false, true><<<grid, 256, 0, stream>>>(p);
    else isp::conv_quant_kernel<false, false><<<grid, 256, 0, stream>>>(p);
  }
  return isp::launch_status();
}

int isp_conv1d(const void* xq, int ab_dtype, int64_t B, int C_pad, int64_t T_in, const void* w_packed, int CO,
               int KW, int stride, int dilation, int padding, int output_padding, int transposed, int64_t T_out,
               float in_scale, const float* amax, const float* w_scale, const float* bias, void* y, int out_dtype,
               isp_stream_t stream) {
  using namespace isp::gemm;
  if (xq == nullptr || w_packed == nullptr || y == nullptr || w_scale == nullptr) return ISP_ERR_ARG;
  if (ab_dtype != ISP_E4M3 && ab_dtype != ISP_I8) return ISP_ERR_DTYPE;
  if (out_dtype != ISP_F32 && out_dtype != ISP_BF16 && out_dtype != ISP_F16) return ISP_ERR_DTYPE;
  if (amax != nullptr ? (ab_dtype != ISP_E4M3 || in_scale != 0.f) : !(in_scale > 0.f)) return ISP_ERR_ARG;
  ConvGeom g;
  if (int st = conv_geometry(KW, stride, dilation, padding, transposed, &g)) return st;
  if (B < 0 || B > 0xFFFF || C_pad <= 0 || C_pad % 128 != 0 || T_in <= 0 || CO <= 0 || output_padding < 0 ||
      T_in > 0x3FFFFFFFll || T_out > 0x3FFFFFFFll)
    return ISP_ERR_SHAPE;
  const int64_t expect = transposed ? (T_in - 1) * stride - 2 * static_cast<int64_t>(padding) +
                                          static_cast<int64_t>(dilation) * (KW - 1) + output_padding + 1
                                    : (T_in + 2 * static_cast<int64_t>(padding) -
                                       static_cast<int64_t>(dilation) * (KW - 1) - 1) / stride + 1;
  if (T_out != expect || T_out <= 0 || (!transposed && output_padding != 0)) return ISP_ERR_SHAPE;
  const int cblocks = C_pad / kBK;
  if (g.a_stride * cblocks > 1023) return ISP_ERR_SHAPE;
  if (!isp::aligned16(xq) || !isp::aligned16(w_packed) || !isp::aligned16(w_scale) ||
      (bias && !isp::aligned16(bias)))
    return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (B == 0) return ISP_OK;
  const int64_t k_bytes = static_cast<int64_t>(g.taps) * C_pad;
  const int64_t t_rows = (T_in + g.a_stride - 1) / g.a_stride;   // rows of the A view per utterance
  const int64_t q_rows = (T_out + g.phases - 1) / g.phases;      // phase rows per utterance
  const int tpb = static_cast<int>((q_rows + kBM - 1) / kBM);
  const int64_t n_cols = static_cast<int64_t>(CO) * g.phases;
  if (k_bytes > 0x7FFFFFFFll || n_cols > 0x7FFFFFFFll || static_cast<int64_t>(B) * tpb * kBM > 0x7FFFFFFFll ||
      static_cast<int64_t>(B) * tpb * ((n_cols + kBN - 1) / kBN) > 0x7FFFFFFFll)
    return ISP_ERR_SHAPE;
  CUtensorMap ta, tb;
  if (!make_map3d_u8(&ta, xq, static_cast<uint64_t>(g.a_stride) * C_pad, static_cast<uint64_t>(t_rows),
                     static_cast<uint64_t>(B), kBK, kBM) ||
      !make_map(&tb, w_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, static_cast<uint64_t>(k_bytes),
                static_cast<uint64_t>(n_cols), kBK, kBN))
    return ISP_ERR_ALIGN;
  Params p{};
  p.conv_tpb = tpb;
  p.conv_phases = g.phases;
  p.conv_taps = g.taps;
  p.conv_cblocks = cblocks;
  p.conv_co = CO;
  p.conv_tout = T_out;
  p.conv_amax = amax;
  for (int j = 0; j < g.taps; ++j) p.conv_tab[j] = g.row[j] * 1024 + g.colstep[j] * cblocks;
  p.M = static_cast<int>(B * tpb * kBM);
  p.N = static_cast<int>(n_cols);
  p.K = static_cast<int>(k_bytes);
  p.m_tiles = static_cast<int>(B * tpb);
  p.n_tiles = static_cast<int>((n_cols + kBN - 1) / kBN);
  p.k_blocks = g.taps * cblocks;
  p.a_scale = amax != nullptr ? 1.f : in_scale;   // dynamic: the epilogue applies the utterance's scale
  p.w_scale = w_scale;
  p.bias = bias;
  p.out = y;
  // Output boxes through a tensor map where its rules allow (row pitch a multiple of
  // 16 bytes, at most 8 phases); otherwise per-element stores.
  const int out_kind = out_dtype == ISP_F32 ? OUT_F32 : (out_dtype == ISP_F16 ? OUT_F16 : OUT_BF16);
  CUtensorMap to = ta;
  p.conv_tma_store = (g.phases == 1 || g.phases == 2 || g.phases == 4 || g.phases == 8) &&
                     (T_out * out_bytes(out_kind)) % 16 == 0 && !conv_direct_forced() &&
                     make_conv_out_map(&to, y, out_kind, static_cast<uint64_t>(T_out), static_cast<uint64_t>(CO),
                                       static_cast<uint64_t>(B), static_cast<uint32_t>(g.phases));
  const bool stat = k_bytes <= kStatK && !streaming_forced();
  if (ab_dtype == ISP_I8) {
    switch (out_dtype) {
      case ISP_F32: return launch_conv<AB_I8, OUT_F32>(stat, ta, tb, to, p, stream);
      case ISP_F16: return launch_conv<AB_I8, OUT_F16>(stat, ta, tb, to, p, stream);
      default: return launch_conv<AB_I8, OUT_BF16>(stat, ta, tb, to, p, stream);
    }
  }
  switch (out_dtype) {
    case ISP_F32: return launch_conv<AB_E4M3, OUT_F32>(stat, ta, tb, to, p, stream);
    case ISP_F16: return launch_conv<AB_E4M3, OUT_F16>(stat, ta, tb, to, p, stream);
    default: return launch_conv<AB_E4M3, OUT_BF16>(stat, ta, tb, to, p, stream);
  }
}

int isp_fir_snake(const float* x, int64_t rows, int C, int64_t T, const float* up,
                  const float* down, const float* alpha, const float* inv_beta, void* y,
                  int out_dtype, const float* smooth, float scale, isp_stream_t stream) {
  if (!x || !up || !down || !alpha || !inv_beta || !y) return ISP_ERR_ARG;
  if (out_dtype != ISP_F32 && out_dtype != ISP_I8) return ISP_ERR_DTYPE;
  if (out_dtype == ISP_I8 && (smooth == nullptr || !(scale > 0.f))) return ISP_ERR_ARG;
  if (rows < 0 || C <= 0 || T <= 0 || (rows % C) != 0) return ISP_ERR_SHAPE;
  if (T > (int64_t(1) << 40) || rows > 0x7FFFFFFFll) return ISP_ERR_SHAPE;
  if (!isp::aligned16(x) || (out_dtype == ISP_F32 && (reinterpret_cast<uintptr_t>(y) & 7))) return ISP_ERR_ALIGN;
  const bool bulk = T % 4 == 0;                         // rows fetched in 16-byte granules
  if (int st = isp::check_device()) return st;
  if (rows == 0) return ISP_OK;
  const int64_t tiles = (T + isp::kFirTile - 1) / isp::kFirTile;
  isp::FirParams p{};
  p.x = x;
  p.rows = rows;
  p.C = C;
  p.T = T;
  p.tiles_per_row = tiles;
  p.alpha = alpha;
  p.inv_beta = inv_beta;
  p.y = y;
  p.smooth = smooth;
  p.scale = scale;
  for (int k = 0; k < 12; ++k) {   // host arrays: the taps travel by value
    p.up2[k] = 2.f * up[k];
    p.down[k] = down[k];
  }
  for (int m = 0; m < 6; ++m) p.upp[m] = make_float2(p.up2[11 - 2 * m], p.up2[10 - 2 * m]);
  for (int k = 0; k < 5; ++k) p.dnp[k] = make_float2(p.down[2 * k + 1], p.down[2 * k + 2]);
  p.rscale = 1.f / scale;   // RN(1/s) (IEEE single-precision division on the host)
  auto kern = out_dtype == ISP_F32 ? (bulk ? isp::fir_snake_kernel<false, true> : isp::fir_snake_kernel<false, false>)
                                   : (bulk ? isp::fir_snake_kernel<true, true> : isp::fir_snake_kernel<true, false>);
  static bool configured[4][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  const int which = (out_dtype == ISP_F32 ? 0 : 2) + (bulk ? 1 : 0);
  if (dev >= 0 && dev < 64 && !configured[which][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, isp::kFirSmemBytes) != cudaSuccess)
      return ISP_ERR_LAUNCH;
    configured[which][dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, isp::kFirThreads, isp::kFirSmemBytes) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t total = rows * tiles;
  const int64_t cap = static_cast<int64_t>(isp::sm_count()) * per_sm;
  const unsigned grid = static_cast<unsigned>(total < cap ? total : cap);
  p.g_rows = static_cast<int>(grid / tiles);
  p.g_tiles = static_cast<int>(grid % tiles);
  p.g_chan = p.g_rows % C;
  kern<<<grid, isp::kFirThreads, isp::kFirSmemBytes, stream>>>(p);
  return isp::launch_status();
}

int isp_scaled_gemm(const void* A, const void* W, int ab_dtype, int64_t M, int N, int K, float a_scale,
                    const float* a_scale_rows, const float* w_scale, const float* bias, const void* residual,
                    int residual_dtype, void* out, int out_dtype, float out_inv_scale, void* out2,
                    float out2_inv_scale, isp_stream_t stream) {
  using namespace isp::gemm;
  if (A == nullptr || W == nullptr || out == nullptr) return ISP_ERR_ARG;
  if (ab_dtype != ISP_E4M3 && ab_dtype != ISP_I8) return ISP_ERR_DTYPE;
  const int out_kind = out_kind_of(out_dtype);
  if (out_kind < 0) return ISP_ERR_DTYPE;
  if (residual != nullptr && residual_dtype != ISP_F32 && residual_dtype != ISP_BF16) return ISP_ERR_DTYPE;
  if (M < 0 || M > 0x7FFFFFFFll || N <= 0 || K <= 0 || K % 16 != 0 || N % 16 != 0) return ISP_ERR_SHAPE;
  if (!isp::aligned16(A) || !isp::aligned16(W) || !isp::aligned16(out)) return ISP_ERR_ALIGN;
  if ((w_scale && !isp::aligned16(w_scale)) || (bias && !isp::aligned16(bias)) || (out2 && !isp::aligned16(out2)))
    return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (M == 0) return ISP_OK;
  if (M <= kBM && out2 == nullptr && out_kind != OUT_E4M3 && !decode_disabled()) {
    // decode: one 128-column N tile per cluster, K split over up to 8 CTAs
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, kBK, kBM) ||
        !make_map(&tb, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, kBK, kDecBN))
      return ISP_ERR_ALIGN;
    Params p{};
    p.M = static_cast<int>(M);
    p.N = N;
    p.K = K;
    p.k_blocks = (K + kBK - 1) / kBK;
    p.a_scale = a_scale;
    p.a_scale_rows = a_scale_rows;
    p.w_scale = w_scale;
    p.bias = bias;
    p.residual = residual;
    p.residual_f32 = residual_dtype == ISP_F32;
    p.out = out;
    const int n_tiles = (N + kDecBN - 1) / kDecBN;
    int splits = kDecMaxSplits;
    while (splits > 1 && (n_tiles * splits > isp::sm_count() || splits > p.k_blocks)) splits >>= 1;
    return ab_dtype == ISP_I8 ? dispatch_decode<true>(out_kind, ta, tb, p, splits, n_tiles, stream)
                              : dispatch_decode<false>(out_kind, ta, tb, p, splits, n_tiles, stream);
  }
  // K <= 512 bytes: B-stationary, else B streamed through the ring; both on SM pairs
  // (256-row tiles, half of B per SM)
  const bool stat = K <= kStatK && !streaming_forced();
  const int sched = !stat ? (pair_schedule_enabled() ? SCHED_PAIR_STREAM : SCHED_STREAM)
                          : (pair_schedule_enabled() ? SCHED_PAIR : SCHED_STAT);
  CUtensorMap ta, tb, to;
  if (!make_map(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, kBK, kBM) ||
      !make_map(&tb, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, kBK, sched_pair(sched) ? kBN / 2 : kBN) ||
      !make_out_map(&to, out, out_kind, M, N))
    return ISP_ERR_ALIGN;
  Params p{};
  p.M = static_cast<int>(M);
  p.N = N;
  p.K = K;
  p.m_tiles = static_cast<int>((M + (sched_pair(sched) ? 2 * kBM : kBM) - 1) / (sched_pair(sched) ? 2 * kBM : kBM));
  p.n_tiles = (N + kBN - 1) / kBN;
  p.k_blocks = (K + kBK - 1) / kBK;
  p.a_scale = a_scale;
  p.a_scale_rows = a_scale_rows;
  p.w_scale = w_scale;
  p.bias = bias;
  p.residual = residual;
  p.residual_f32 = residual_dtype == ISP_F32;
  p.out_inv = out_inv_scale;
  p.out2 = out2;
  p.out2_inv = out2_inv_scale;
  // streaming: the last partial wave runs as half-N tiles (needs the two-warps-per-quarter
  // epilogue, whose upper warps simply hand a half tile's accumulator back)
  // (single CTAs only: an SM pair's tile is not split)
  p.tail_split = sched == SCHED_STREAM && kScaleEpiWarps == 8 && !tail_split_disabled();
  return ab_dtype == ISP_I8 ? dispatch_scale_out<AB_I8>(out_kind, sched, ta, tb, to, p, stream)
                            : dispatch_scale_out<AB_E4M3>(out_kind, sched, ta, tb, to, p, stream);
}

int isp_gated_up(const void* A, const void* W1, const void* W3, int interleaved, int64_t M, int N, int K,
                 const float* s1, const float* s3, float out_scale, void* out, int out_dtype,
                 isp_stream_t stream) {
  using namespace isp::gemm;
  if (A == nullptr || W1 == nullptr || s1 == nullptr || out == nullptr) return ISP_ERR_ARG;
  if (interleaved ? (W3 != nullptr || s3 != nullptr) : (W3 == nullptr || s3 == nullptr)) return ISP_ERR_ARG;
  if (out_dtype != ISP_E4M3 && out_dtype != ISP_F32) return ISP_ERR_DTYPE;
  if (!(out_scale > 0.f)) return ISP_ERR_ARG;
  if (M < 0 || M > 0x7FFFFFFFll || N <= 0 || K <= 0 || K % 16 != 0 || N % 32 != 0) return ISP_ERR_SHAPE;
  if (!isp::aligned16(A) || !isp::aligned16(W1) || !isp::aligned16(out) || !isp::aligned16(s1) ||
      (W3 && !isp::aligned16(W3)) || (s3 && !isp::aligned16(s3)))
    return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (M == 0) return ISP_OK;
  const int out_kind = out_dtype == ISP_E4M3 ? OUT_E4M3 : OUT_F32;
  CUtensorMap ta, tb, tb2, to;
  if (!make_map(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, kBK, kBM) || !make_out_map(&to, out, out_kind, M, N))
    return ISP_ERR_ALIGN;
  if (interleaved) {
    if (!make_map(&tb, W1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, 2ull * N, kBK, kBN)) return ISP_ERR_ALIGN;
    tb2 = tb;
  } else {
    if (!make_map(&tb, W1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, kBK, kBN / 2) ||
        !make_map(&tb2, W3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, kBK, kBN / 2))
      return ISP_ERR_ALIGN;
  }
  Params p{};
  p.M = static_cast<int>(M);
  p.N = N;
  p.K = K;
  p.m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  p.n_tiles = (N + kBN / 2 - 1) / (kBN / 2);
  p.k_blocks = (K + kBK - 1) / kBK;
  p.a_scale = 1.f;
  p.w_scale = s1;
  p.w_scale2 = s3;
  p.out_inv = static_cast<float>(1.0 / static_cast<double>(out_scale));
  p.out_scale = out_scale;
  const bool stat = K <= kStatK && !streaming_forced();
  constexpr int kSt = kStatStages + 1;   // 4 epilogue warps leave room for a fifth A stage
  if (interleaved) {
    if (out_kind == OUT_E4M3)
      return stat ? launch<kBN, kSt, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_INTERLEAVED, OUT_E4M3, kStatK>(ta, tb, tb2, to, p, stream)
                  : launch<kBN, kStages, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_INTERLEAVED, OUT_E4M3>(ta, tb, tb2, to, p, stream);
    return stat ? launch<kBN, kSt, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_INTERLEAVED, OUT_F32, kStatK>(ta, tb, tb2, to, p, stream)
                : launch<kBN, kStages, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_INTERLEAVED, OUT_F32>(ta, tb, tb2, to, p, stream);
  }
  if (out_kind == OUT_E4M3)
    return stat ? launch<kBN, kSt, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_PAIRED, OUT_E4M3, kStatK>(ta, tb, tb2, to, p, stream)
                : launch<kBN, kStages, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_PAIRED, OUT_E4M3>(ta, tb, tb2, to, p, stream);
  return stat ? launch<kBN, kSt, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_PAIRED, OUT_F32, kStatK>(ta, tb, tb2, to, p, stream)
              : launch<kBN, kStages, kSwigluEpiWarps, AB_E4M3, EPI_SWIGLU_PAIRED, OUT_F32>(ta, tb, tb2, to, p, stream);
}

int isp_int8_nonlinear_value(const void* Q, const void* W, int64_t M, int N, int K, int groups, float a_scale,
                             const float* w_scale, const float* bias, float* value, float* gate,
                             isp_stream_t stream) {
  using namespace isp::gemm;
  if (Q == nullptr || W == nullptr || w_scale == nullptr || bias == nullptr || value == nullptr || gate == nullptr)
    return ISP_ERR_ARG;
  if (!(a_scale > 0.f) || a_scale == INFINITY) return ISP_ERR_ARG;
  if (M < 0 || M > 0x7FFFFFFFll || N <= 0 || N % 16 != 0 || N > 0x7FFFFFFF / 3 || K <= 0 || K % 16 != 0 ||
      groups < 1 || M % groups != 0)
    return ISP_ERR_SHAPE;
  if (!isp::aligned16(Q) || !isp::aligned16(W) || !isp::aligned16(w_scale) || !isp::aligned16(bias) ||
      !isp::aligned16(value) || !isp::aligned16(gate))
    return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (M == 0) return ISP_OK;
  CUtensorMap ta, tb;
  if (!make_map(&ta, Q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, kBK, kBM) ||
      !make_map(&tb, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, 3ull * N, kBK, kNlvBN / 3))
    return ISP_ERR_ALIGN;
  Params p{};
  p.M = static_cast<int>(M);
  p.N = N;
  p.K = K;
  p.m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  p.n_tiles = (N + kNlvBN / 3 - 1) / (kNlvBN / 3);
  p.k_blocks = (K + kBK - 1) / kBK;
  p.a_scale = a_scale;
  p.w_scale = w_scale;
  p.bias = bias;
  p.out = value;
  p.nlv_gate = gate;
  p.nlv_groups = groups;
  // The output map is unused (direct stores); pass Q's.
  if (K <= kStatK)
    return launch<kNlvBN, kNlvStatStages, 8, AB_I8, EPI_NLV, OUT_F32, kStatK>(ta, tb, tb, ta, p, stream);
  return launch<kNlvBN, kStages, 8, AB_I8, EPI_NLV, OUT_F32>(ta, tb, tb, ta, p, stream);
}

int isp_nvfp4_scales_to_mma(const void* src, int64_t R, int K, void* dst, isp_stream_t stream) {
  if (src == nullptr || dst == nullptr) return ISP_ERR_ARG;
  if (R < 0 || K <= 0 || K % 64 != 0 || R > (int64_t(1) << 40)) return ISP_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(src) & 3) || (reinterpret_cast<uintptr_t>(dst) & 3)) return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (R == 0) return ISP_OK;
  const int kchunks = K / 64;
  const int64_t words = (R + 127) / 128 * 128 * kchunks;
  const unsigned grid = static_cast<unsigned>((words + 255) / 256);
  isp::gemm::scales_to_mma_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint32_t*>(src), R, kchunks,
                                                           static_cast<uint32_t*>(dst), words);
  return isp::launch_status();
}

int isp_nvfp4_gemm(const void* A, const void* A_sf, const void* W, const void* W_sf, int64_t M, int N, int K,
                   float alpha, const float* bias, const void* residual, int residual_dtype, void* out, int out_dtype,
                   isp_stream_t stream) {
  using namespace isp::gemm;
  if (!A || !A_sf || !W || !W_sf || !out) return ISP_ERR_ARG;
  if (out_dtype != ISP_BF16 && out_dtype != ISP_F16 && out_dtype != ISP_F32) return ISP_ERR_DTYPE;
  if (residual != nullptr && residual_dtype != ISP_F32 && residual_dtype != ISP_BF16) return ISP_ERR_DTYPE;
  if (!(alpha == alpha) || alpha == INFINITY || alpha == -INFINITY) return ISP_ERR_ARG;
  if (M < 0 || M > 0x7FFFFFFFll || N <= 0 || K <= 0 || K % 64 != 0 || N % 8 != 0) return ISP_ERR_SHAPE;
  if (!isp::aligned16(A) || !isp::aligned16(W) || !isp::aligned16(A_sf) || !isp::aligned16(W_sf) ||
      !isp::aligned16(out) || (bias && !isp::aligned16(bias)))
    return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (M == 0) return ISP_OK;
  const int out_kind = out_kind_of(out_dtype);
  CUtensorMap ta, tb, to;
  if (!make_map(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, M, kBK, kBM) ||
      !make_map(&tb, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, kBK, kFp4BN) ||
      !make_out_map(&to, out, out_kind, M, N))
    return ISP_ERR_ALIGN;
  Params p{};
  p.M = static_cast<int>(M);
  p.N = N;
  p.K = K;
  p.m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  p.n_tiles = (N + kFp4BN - 1) / kFp4BN;
  p.k_blocks = (K / 2 + kBK - 1) / kBK;
  p.k_chunks = K / 64;
  p.sfa = static_cast<const uint8_t*>(A_sf);
  p.sfb = static_cast<const uint8_t*>(W_sf);
  p.a_scale = alpha;
  p.bias = bias;
  p.residual = residual;
  p.residual_f32 = residual_dtype == ISP_F32;
  const bool stat = K / 2 <= kStatK && !streaming_forced();
  return dispatch_scale_out<AB_FP4>(out_kind, stat ? SCHED_STAT : SCHED_STREAM, ta, tb, to, p, stream);
}

int isp_nvfp4_gated_up(const void* A, const void* A_sf, const void* W13, const void* W13_sf, int64_t M, int N, int K,
                       float alpha_gate, float alpha_up, float h_scale, void* h_codes, void* h_sf,
                       isp_stream_t stream) {
  using namespace isp::gemm;
  if (!A || !A_sf || !W13 || !W13_sf || !h_codes || !h_sf) return ISP_ERR_ARG;
  if (!(alpha_gate == alpha_gate) || !(alpha_up == alpha_up) || alpha_gate == INFINITY || alpha_gate == -INFINITY ||
      alpha_up == INFINITY || alpha_up == -INFINITY || !global_scale_ok(h_scale))
    return ISP_ERR_ARG;
  if (M < 0 || M > 0x7FFFFFFFll || N <= 0 || K <= 0 || K % 64 != 0 || N % 64 != 0) return ISP_ERR_SHAPE;
  if (!isp::aligned16(A) || !isp::aligned16(W13) || !isp::aligned16(A_sf) || !isp::aligned16(W13_sf) ||
      !isp::aligned16(h_codes) || !isp::aligned16(h_sf))
    return ISP_ERR_ALIGN;
  if (int st = isp::check_device()) return st;
  if (M == 0) return ISP_OK;
  CUtensorMap ta, tb;
  if (!make_map(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, M, kBK, kBM) ||
      !make_map(&tb, W13, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, 2ull * N, kBK, kFp4BN))
    return ISP_ERR_ALIGN;
  Params p{};
  p.M = static_cast<int>(M);
  p.N = N;
  p.K = K;
  p.m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  p.n_tiles = N / (kFp4BN / 2);
  p.k_blocks = (K / 2 + kBK - 1) / kBK;
  p.k_chunks = K / 64;
  p.sfa = static_cast<const uint8_t*>(A_sf);
  p.sfb = static_cast<const uint8_t*>(W13_sf);
  p.a_scale = alpha_gate;
  p.alpha_up = alpha_up;
  p.q_scale = h_scale;
  p.q_codes = static_cast<uint8_t*>(h_codes);
  p.q_sf = static_cast<uint8_t*>(h_sf);
  // The output map is unused by the NVFP4 epilogue (direct stores); pass A's.
  if (K / 2 <= kStatK && !streaming_forced())
    return launch<kFp4BN, kFp4StatStages + 2, kFp4SwigluEpiWarps, AB_FP4, EPI_SWIGLU_PAIRED, OUT_NVFP4, kStatK>(
        ta, tb, tb, ta, p, stream);
  return launch<kFp4BN, kFp4Stages, kFp4SwigluEpiWarps, AB_FP4, EPI_SWIGLU_PAIRED, OUT_NVFP4>(ta, tb, tb, ta, p,
                                                                                          stream);
}

// ---- dynamic-scale convolution without caller scratch (array above extern "C") ----
int isp_conv1d_dynamic_noalloc(const void* x, int x_dtype, int64_t B, int C, int64_t T, void* xq, int C_pad,
                               const void* w_packed, int CO, int KW, int stride, int dilation, int padding,
                               int output_padding, int transposed, int64_t T_out, const float* w_scale,
                               const float* bias, void* y, int out_dtype, isp_stream_t stream) {
  if (B > kConvNoAllocMaxBatch) return ISP_ERR_SHAPE;   // more utterances than the scratch holds
  if (x == nullptr || xq == nullptr || w_packed == nullptr || w_scale == nullptr || y == nullptr) return ISP_ERR_ARG;
  if (B < 0) return ISP_ERR_SHAPE;
  if (int st = isp::check_device()) return st;
  // Scratch address of the current device, resolved on that device's first call.
  static float* amax_of[64] = {nullptr};
  static std::mutex setup;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ISP_ERR_ARCH;
  float* amax = nullptr;
  {
    std::lock_guard<std::mutex> lock(setup);
    if (amax_of[dev] == nullptr) {
      void* addr = nullptr;
      if (cudaGetSymbolAddress(&addr, g_conv_amax_scratch) != cudaSuccess || addr == nullptr) return ISP_ERR_LAUNCH;
      amax_of[dev] = static_cast<float*>(addr);
    }
    amax = amax_of[dev];
  }
  // isp_conv1d_quant clears amax[0 .. B) before its maximum pass
  const int row_multiple = transposed ? 1 : stride;
  if (int st = isp_conv1d_quant(x, x_dtype, B, C, T, row_multiple, nullptr, 0.f, amax, ISP_E4M3, xq, C_pad, stream))
    return st;
  return isp_conv1d(xq, ISP_E4M3, B, C_pad, T, w_packed, CO, KW, stride, dilation, padding, output_padding,
                    transposed, T_out, 0.f, amax, w_scale, bias, y, out_dtype, stream);
}

}  // extern "C"
