// Shared device/host helpers for the sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/isp_b200.h"

#define ISP_HD __host__ __device__ __forceinline__
#define ISP_D __device__ __forceinline__

namespace isp {

// ---------------------------------------------------------------------------
// Host-side validation helpers
// ---------------------------------------------------------------------------
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Checks (once per device) that the current device is compute capability 10.x.
int check_device();
// Multiprocessor count of the current device (cached per device).
int sm_count();

// Maps the last CUDA launch error to a status code (clears sticky launch error).
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ISP_OK : ISP_ERR_LAUNCH;
}

// Launch with programmatic stream serialization: the kernel may be scheduled while
// its predecessor in the stream finishes, and must call pdl_wait() before touching
// global memory.  Returns an isp_status.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  (void)cudaGetLastError();   // the status is returned here, not left for a later launch_status()
  return e == cudaSuccess ? ISP_OK : ISP_ERR_LAUNCH;
}

// launch_pdl for a kernel of thread-block clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
inline int launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              unsigned cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  (void)cudaGetLastError();
  return e == cudaSuccess ? ISP_OK : ISP_ERR_LAUNCH;
}

// Device error word (one per device; the library is a single translation unit).
__device__ int g_device_error = 0;

// ---------------------------------------------------------------------------
// Number formats (device).  E4M3 conversion uses the hardware cvt with
// round-to-nearest-even and saturation to +-448 (NaN stays NaN).
// ---------------------------------------------------------------------------
// Packs two floats into two E4M3 bytes: `lo` goes to bits 0-7, `hi` to 8-15.
ISP_D uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

ISP_D float e4m3_to_f32(uint8_t code) {
  uint16_t packed = code;
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(packed));
  __half h = __ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu));
  return __half2float(h);
}

ISP_D float clamp448(float v) { return fminf(fmaxf(v, -448.f), 448.f); }

// E2M1 code (sign in bit 3) of v: midpoints go to the even code, magnitudes
// above 6 saturate, the sign bit is (v < 0).  Written from the format
// definition; decision points 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.
ISP_D uint32_t e2m1_code(float v) {
  float a = fabsf(v);
  uint32_t m = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) +
               (a >= 3.5f) + (a > 5.0f);
  return m | (v < 0.f ? 8u : 0u);
}

// Two E2M1 codes from the hardware conversion (round to nearest even,
// saturating to +-6): `lo` in bits 0-3, `hi` in bits 4-7.  Matches e2m1_code
// on every finite input except -0.0 (hardware: 0x8); callers pass +-0 as +0.
ISP_D uint32_t e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n cvt.u32.u8 %0, t;\n}" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// RN(x / d) from a reciprocal y = RN(1/d) shared by many quotients (one
// reciprocal per scale instead of one division per element).  Markstein's
// correction (P. Markstein, IBM J. Res. Dev. 34(1), 1990; Muller et al.,
// "Handbook of Floating-Point Arithmetic", ch. 4): q = RN(x y), the residual
// r = x - q d is exact in one FMA, and RN(q + r y) is the correctly rounded
// quotient when y is the correctly rounded reciprocal and q is within one ulp
// (Markstein's theorem; one correction step).  Exact for normal d below 2^126
// and normal quotients (a subnormal quotient can differ by one subnormal ulp,
// below every code's resolution); when the first product is out of range
// (|q| >= 2^100, inf, NaN) or d is zero or at least 2^126, x * y is returned,
// which equals x / d up to the saturation every caller applies next (inf, NaN
// and 0 propagate as in x / d).
ISP_D float div_rn_recip(float x, float d, float y) {
  const float q0 = __fmul_rn(x, y);
  const float r = __fmaf_rn(-q0, d, x);
  const float q = __fmaf_rn(r, y, q0);
  return (fabsf(q0) < 0x1p100f && fabsf(d) < 0x1p126f) ? q : q0;
}

// div_rn_recip on two quotients with one divisor, the three IEEE steps two lanes per
// instruction (f32x2: each lane rounded exactly as the scalar operation).
ISP_D float2 div_rn_recip2(float2 x, float d, float y) {
  const float2 q0 = __fmul2_rn(x, make_float2(y, y));
  const float2 r = __ffma2_rn(q0, make_float2(-d, -d), x);
  const float2 q = __ffma2_rn(r, make_float2(y, y), q0);
  const bool dd = fabsf(d) < 0x1p126f;
  return make_float2((fabsf(q0.x) < 0x1p100f && dd) ? q.x : q0.x, (fabsf(q0.y) < 0x1p100f && dd) ? q.y : q0.y);
}

ISP_D int8_t int8_rne_sat(float v) {
  int q = __float2int_rn(v);
  q = q < -128 ? -128 : (q > 127 ? 127 : q);
  return static_cast<int8_t>(q);
}

ISP_D float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while its predecessor in the stream is still running;
// pdl_wait() blocks until that predecessor has completed and its writes are visible
// (a no-op for an ordinary launch), so no global memory may be read or written
// before it.  pdl_trigger() lets the next such kernel start its own prologue.
ISP_D void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
ISP_D void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// RN to BF16 of (lo, hi) in one conversion: lo in bits 0-15, hi in bits 16-31.
ISP_D uint32_t pack_bf16_rn(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// Global-memory vector helpers
// ---------------------------------------------------------------------------
ISP_D uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

ISP_D void bf16x8_to_f32(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// ---------------------------------------------------------------------------
// Bounded waits: every spin gives up after ~1 s of %globaltimer, records
// ISP_ERR_TIMEOUT in g_device_error and reports failure to the caller, which
// then unwinds without touching the data path.
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitLimitNs = 1000000000ull;

ISP_D uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

ISP_D void record_timeout() { atomicExch(&g_device_error, (int)ISP_ERR_TIMEOUT); }

}  // namespace isp
