// W8A8 (E4M3 / INT8) and NVFP4 GEMM on 5th-generation tensor cores (tcgen05),
// sm_100a.
//
// out[M, N] = epilogue(A[M, K] . B[N, K]^T), both operands K-major: 8-bit codes
// (kind::f8f6f4 / kind::i8), or packed E2M1 with one E4M3 scale per 16 K
// (kind::mxf4nvf4.block_scale.block16).  A stage always holds 128 bytes of K
// per row (128 8-bit or 256 4-bit elements).
//
// Persistent, warp-specialized CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: A and B tiles (BK = 128 bytes of K, 128-byte
//               swizzle) into a kStages-deep shared-memory ring.
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues
//               tcgen05.mma (M = 128, N = BN, K = 32 per instruction) into one
//               of two TMEM accumulators, so the epilogue of tile i overlaps
//               the main loop of tile i+1.
//   warps 2..   epilogue: tcgen05.ld (32 lanes x 32 columns per load), fused
//               scale / bias / residual / SwiGLU / requant, 128-byte swizzled
//               staging and TMA stores (NVFP4 outputs: direct 16-byte stores).
// NVFP4 adds the block scales: each stage carries 2 KB of A scales and 2 KB of
// B scales (four 512-byte chunks of 128 rows x 4 scales each, copied in the
// tensor-core layout by one bulk copy per operand), which the MMA thread moves
// into TMEM with tcgen05.cp (32 lanes x 128 bits, replicated to the 4 lane
// quarters) right before the four K = 64 MMAs that read them.
// Every mbarrier wait is bounded (~1 s); on expiry the waiting thread records
// ISP_ERR_TIMEOUT in g_device_error, raises the CTA abort flag, and all roles
// unwind to the common exit.  The producer and MMA warps first wait (ignoring the
// flag, bounded by their own limit) for the loads and MMAs they issued; then TMEM
// is freed.
#pragma once

#include "common.cuh"

namespace isp {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 128;          // bytes (= elements) of K per stage
constexpr int kEpiWarp0 = 2;      // warps 0 (TMA) and 1 (MMA) precede the epilogue warps

// 32-row x 128-byte store boxes per epilogue warp: one on a single SM (its shared
// memory holds the whole B tile), two on SM pairs (half of B per SM), so a warp
// writes its next box while the previous one is still being read by the TMA store.
constexpr int kStagingBufsOne = 1;
constexpr int kStagingBufsPair = 2;

// 4 epilogue warps cover the 4 TMEM lane quarters once; 8 warps take two per
// quarter, each on half of the tile's columns (twice the latency hiding).
template <int kEpiWarps>
struct Roles {
  static constexpr int kEpiThreads = kEpiWarps * 32;
  static constexpr int kThreads = 64 + kEpiThreads;
  static constexpr int kHalves = kEpiWarps / 4;
};
// NVFP4 kernels add one warp after the epilogue warps that copies each stage's block
// scales into TMEM (tcgen05.cp costs the issuing thread ~115 cycles, more than the
// K = 64 MMA it feeds), so the MMA warp issues only MMAs.
template <int kEpiWarps, bool kFp4>
constexpr int kernel_threads() { return Roles<kEpiWarps>::kThreads + (kFp4 ? 32 : 0); }

enum AbKind { AB_E4M3 = 0, AB_I8 = 1, AB_FP4 = 2 };
// EPI_CONV: the scale epilogue of a phase-folded implicit-GEMM convolution (A rows =
// phase rows of one utterance, A gathered per (window slot, 128-channel) block from
// channels-last codes; column co * P + r is output channel co at phase r; output
// stored transposed to [B, CO, T_out]).
// EPI_NLV: the INT8 nonlinear-value projection: one tile = 64 outputs x 3 stacked
// projections (B rows [0, 64) = W[n0 ..], [64, 128) = W[N + n0 ..], [128, 192) =
// W[2N + n0 ..]); z_j = acc_j * (AS * WS[jN + n]) + bias[jN + n], stored as
// value = tanh(z0) * z1 (rows re-ordered from (t, b) to (b, t)) and gate = z2.
enum EpiKind { EPI_SCALE = 0, EPI_SWIGLU_PAIRED = 1, EPI_SWIGLU_INTERLEAVED = 2, EPI_CONV = 3, EPI_NLV = 4 };
constexpr int kNlvBN = 192;   // EPI_NLV tile: 3 x 64 accumulator columns
// OUT_NVFP4: packed E2M1 codes + E4M3 block scales in the tensor-core layout.
enum OutKind { OUT_BF16 = 0, OUT_F16 = 1, OUT_F32 = 2, OUT_E4M3 = 3, OUT_NVFP4 = 4 };

ISP_HD int out_bytes(int out) { return out == OUT_F32 ? 4 : ((out == OUT_E4M3 || out == OUT_NVFP4) ? 1 : 2); }

constexpr int kSfChunk = 512;                        // 128 rows x 4 E4M3 scales (K = 64)
constexpr int kSfOperandBytes = 4 * kSfChunk;        // one operand's scales for a 256-element K stage
constexpr int kSfStageBytes = 2 * kSfOperandBytes;   // A and B scales of one stage
constexpr int kConvTab = 128;                        // (phase, tap) entries of an implicit conv

// Dynamic per-utterance input scale of the FP8 implicit conv: max(amax / 448, 1e-12).
ISP_D float conv_dynamic_scale(float amax) { return fmaxf(__fdiv_rn(amax, 448.f), 1e-12f); }

struct Params {
  int M, N, K;            // N = logical output columns
  int m_tiles, n_tiles, k_blocks;
  float a_scale;
  const float* a_scale_rows;
  const float* w_scale;   // [N] scale (EPI_SCALE), s1 [N] or interleaved S [2N]
  const float* w_scale2;  // s3 [N] (paired SwiGLU)
  const float* bias;
  const void* residual;
  int residual_f32;
  float out_inv;          // E4M3 output multiplier
  float out_scale;        // SwiGLU dequant multiplier (F32 output)
  void* out2;             // residual-dual E4M3 output
  float out2_inv;
  void* out;              // output base (direct-store paths; TMA stores use the tensor map)
  // NVFP4 operands: block scales of A and B in the tensor-core layout
  // (chunk (r/128, k/64) of 512 bytes at ((r/128) * k_chunks + k/64) * 512).
  const uint8_t* sfa;
  const uint8_t* sfb;
  int k_chunks;           // K / 64
  float alpha_up;         // NVFP4 SwiGLU: up-projection dequant (gate: a_scale)
  float q_scale;          // NVFP4 output: global scale of h
  uint8_t* q_codes;       // NVFP4 output: packed E2M1 [M, N/2]
  uint8_t* q_sf;          // NVFP4 output: block scales, tensor-core layout
  // EPI_CONV (phase-folded implicit-GEMM Conv1d / ConvTranspose1d, P = conv_phases):
  //   m tile mt -> utterance mt / conv_tpb, first phase row q0 = (mt % conv_tpb) * 128;
  //   column n (N = CO * P) -> output channel n / P, phase r = n % P; phase row q of
  //   phase r is output time q * P + r;
  //   K block kb -> window slot j = kb / conv_cblocks, e = conv_tab[j]: the A box starts
  //   at row q0 + (e >> 10) and 128-byte column ((e & 1023) + kb % conv_cblocks).
  int conv_tpb;
  int conv_phases;
  int conv_taps;
  int conv_cblocks;
  int conv_co;
  int64_t conv_tout;
  const float* conv_amax; // per-utterance |x| max (dynamic input scale) or nullptr
  int conv_tma_store;     // 1: output blocks of 32 rows x 32 columns leave through the
                          // [B, CO, T_out] tensor map (boxes of 32/P channels x 32P times)
  int conv_tab[kConvTab];
  // Streaming scale epilogue: run the last partial wave as half-N tiles (two per tile)
  int tail_split;
  // EPI_NLV: gate output [M, N] (FP32; value goes to `out`), rows per time step
  float* nlv_gate;
  int nlv_groups;
};

// Shared-memory layout.  Streaming (kBStatK == 0): stage s = [A | B | A scales | B scales].
// B-stationary (kBStatK > 0 bytes of K): stage s = [A | A scales], then the resident
// B tile (kBStatK / 128 boxes of kBN rows x 128 B) and its scales, loaded once per
// N tile.  Scales exist for NVFP4 only; every swizzled region starts 1024-aligned.
template <int kBN, int kStages, int kEpiWarps, bool kFp4, bool kStaging, int kBStatK, int kStagingBufs = kStagingBufsOne>
struct Smem {
  static constexpr bool kStat = kBStatK > 0;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = kBN * kBK;
  static constexpr int kSf = kFp4 ? kSfOperandBytes : 0;
  static constexpr int kStageBytes = kStat ? kABytes + kSf : kABytes + kBBytes + 2 * kSf;
  static constexpr int a(int s) { return s * kStageBytes; }
  static constexpr int b(int s) { return s * kStageBytes + kABytes; }                 // streaming
  static constexpr int sfa(int s) { return s * kStageBytes + kABytes + (kStat ? 0 : kBBytes); }
  static constexpr int sfb(int s) { return sfa(s) + kSf; }                             // streaming
  static constexpr int kBResOffset = kStages * kStageBytes;
  static constexpr int kBResBytes = kStat ? kBN * kBStatK : 0;
  static constexpr int kSfbResOffset = kBResOffset + kBResBytes;
  static constexpr int kSfbResBytes = (kStat && kFp4) ? (2 * kBStatK / 64) * kSfChunk : 0;
  static constexpr int kStagingOffset = kSfbResOffset + kSfbResBytes;
  // per epilogue warp: buffers of 32 rows x 128 B for the TMA stores (none for direct-store epilogues)
  static constexpr int kStagingBytes = kStaging ? kEpiWarps * kStagingBufs * 32 * 128 : 0;
  static constexpr int kParamOffset = kStagingOffset + kStagingBytes;
  static constexpr int kParamBytes = 512 * 4;              // per-tile column scales / bias
  static constexpr int kBarOffset = kParamOffset + kParamBytes;
  static constexpr int kBytes = kBarOffset + (kFp4 ? 384 : 256);   // + barriers/flags (base is 1024-aligned)
  static_assert(kStageBytes % 1024 == 0 && kBResOffset % 1024 == 0 && kStagingOffset % 1024 == 0,
                "swizzled regions start 1024-byte aligned");
};

// ----------------------------------------------------------------------------
// PTX wrappers
// ----------------------------------------------------------------------------
ISP_D uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

ISP_D void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
ISP_D void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
ISP_D void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
ISP_D bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true on success; false after the time limit or when another
// role of this CTA has already given up (abort flag).
ISP_D bool wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                        uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - start > limit_ns) {
        record_timeout();
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Bounded wait for a converged warp: every lane polls, lane 0's result decides,
// and the warp leaves together (a lone polling lane whose warp-mates are parked
// at a block barrier throttles the tcgen05 issue stream it feeds).
ISP_D bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint64_t limit_ns = kWaitLimitNs) {
  if (__shfl_sync(0xffffffffu, static_cast<int>(mbar_try_wait(bar, parity)), 0)) return true;
  const uint64_t start = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (__shfl_sync(0xffffffffu, static_cast<int>(mbar_try_wait(bar, parity)), 0)) return true;
    if ((i & 63u) == 0) {
      int stop = 0;
      if ((threadIdx.x & 31) == 0) {
        if (*abort_flag) {
          stop = 1;
        } else if (globaltimer() - start > limit_ns) {
          record_timeout();
          *abort_flag = 1;
          stop = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
  }
}

// Drain wait for a converged warp.  In-flight TMA copies and issued tcgen05 MMAs
// complete on their own, so a CTA that is unwinding must still wait for them
// before it retires or frees TMEM: this wait ignores the abort flag and gives up
// only after its own time limit (recording ISP_ERR_TIMEOUT).
ISP_D bool wait_warp_drain(uint64_t* bar, uint32_t parity) {
  if (__shfl_sync(0xffffffffu, static_cast<int>(mbar_try_wait(bar, parity)), 0)) return true;
  const uint64_t start = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (__shfl_sync(0xffffffffu, static_cast<int>(mbar_try_wait(bar, parity)), 0)) return true;
    if ((i & 63u) == 0) {
      int stop = 0;
      if ((threadIdx.x & 31) == 0 && globaltimer() - start > kWaitLimitNs) {
        record_timeout();
        stop = 1;
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
  }
}

ISP_D void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
ISP_D void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// L2 policies: output tiles are written once and never re-read by the same launch
// (evict first); the activation tiles of an SM-pair launch are re-read for every
// column tile of a row block (evict last), so the output stream should not push
// them out of L2 between those reads.
ISP_D uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
ISP_D uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
ISP_D void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "l"(policy_evict_first())
               : "memory");
}
// 1-D bulk copy global -> shared, completing on an mbarrier (16-byte aligned, size % 16 == 0).
ISP_D void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
ISP_D void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
ISP_D void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
ISP_D void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
ISP_D void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
ISP_D void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
ISP_D void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
ISP_D void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

ISP_D void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ISP_D void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile, 128-byte rows, 128-byte swizzle, 8-row groups 1024 B apart.
ISP_D uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);   // start address
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                  // 128-byte swizzle
  return d;
}

// Scale-factor chunk in shared memory: 32 rows x 16 bytes, no swizzle; the
// 8-row core matrices are 128 bytes apart (stride byte offset).
ISP_D uint64_t smem_desc_sf(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (one core matrix along K)
  d |= static_cast<uint64_t>(128 >> 4) << 32;           // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100); layout 0 = no swizzle
  return d;
}

template <int kAB, int kBN, int kM = kBM>
ISP_HD uint32_t instr_desc() {
  if constexpr (kAB == AB_FP4) {
    // Block-scaled descriptor: A/B format E2M1 (1) at bits 7 and 10, scale
    // format UE4M3 (0) at bit 23, scale-factor ids 0, N >> 3 at 17, M >> 4 at 24.
    return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kBN >> 3) << 17) |
           (static_cast<uint32_t>(kBM >> 4) << 24);
  } else {
    // D format (F32 = 1, S32 = 2), A/B format (E4M3 = 0, signed int8 = 1), K-major A and B,
    // N >> 3 at bit 17, M >> 4 at bit 24.
    constexpr bool kInt8 = kAB == AB_I8;
    return (kInt8 ? (2u << 4) : (1u << 4)) | (kInt8 ? (1u << 7) | (1u << 10) : 0u) |
           (static_cast<uint32_t>(kBN >> 3) << 17) | (static_cast<uint32_t>(kM >> 4) << 24);
  }
}

// SMEM -> TMEM copy of one scale chunk: 32 lanes x 128 bits, replicated into
// all four 32-lane quarters (4 TMEM columns).
ISP_D void tmem_cp_sf(uint32_t taddr, uint64_t src_desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc) : "memory");
}

ISP_D void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- clusters and the SM-pair (cta_group::2) forms ----
ISP_D uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster arrives (release) and waits (acquire).
ISP_D void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
ISP_D uint32_t map_to_rank(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
  return r;
}
// Arrive on an mbarrier given by its cluster address (this CTA's or the peer's).
ISP_D void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Arm a barrier given by its cluster address with the bytes this arrive expects.
ISP_D void mbar_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr), "r"(bytes)
               : "memory");
}
// SM-pair tile load: the box lands in this CTA's shared memory and its bytes are
// counted on the barrier at `bar_cluster_addr` (the pair leader's), where the MMA
// that reads both CTAs' halves waits.  No multicast.  kEvictLast: loaded with the
// evict-last L2 policy, for tiles re-read by later tiles of the launch (B-stationary
// A: 2 us less per M = 48640, N = 1536 launch than no hint; streamed weights); the
// streamed A of a K > 512 GEMM (75 MB at M = 48640, K = 1536) is loaded without a hint,
// since evict-last there pushes the next kernel's data out of L2.
template <bool kEvictLast>
ISP_D void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int c0, int c1) {
  if constexpr (kEvictLast) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
        "[%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "l"(policy_evict_last())
        : "memory");
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], "
        "[%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
        : "memory");
  }
}
// Commit of the leader's SM-pair MMAs: one arrive on the barrier at this offset in
// both CTAs of the pair once every MMA issued before it has completed.
ISP_D void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n .reg .b16 m;\n mov.b16 m, 3;\n"
      " tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---- warp-wide forms of the issue helpers: the whole (converged) warp executes them
// with warp-uniform operands and one lane, chosen by elect.sync, issues.  The MMA
// warp's main loop uses these: with the descriptors computed warp-wide instead of
// inside a lane-0 branch, each tcgen05 instruction issues in fewer cycles (measured
// on the NVFP4 gated-up GEMM: 165 -> 148.5 us; FP4 down 79 -> 64.5 us).
#define ISP_ELECT_PRED "elect.sync _|e, 0xffffffff;\n"
ISP_D void tmem_cp_sf_elect(uint32_t taddr, uint64_t src_desc) {
  asm volatile("{\n .reg .pred e;\n " ISP_ELECT_PRED " @e tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n}" ::"r"(
                   taddr),
               "l"(src_desc)
               : "memory");
}
ISP_D void mma_fp4_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                         uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n " ISP_ELECT_PRED
      " @e tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem));
}
// kPair: M = 256 MMA over the SM pair (issued by the leader only): A rows [0, 128) and
// B rows [0, N/2) from the leader's shared memory, A rows [128, 256) and B rows
// [N/2, N) from the peer's, at the same offsets; each CTA's TMEM receives its 128 rows.
template <bool kInt8, bool kPair>
ISP_D void mma_issue_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  if constexpr (kPair && kInt8) {
    asm volatile("{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n " ISP_ELECT_PRED
                 " @e tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else if constexpr (kPair) {
    asm volatile("{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n " ISP_ELECT_PRED
                 " @e tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else if constexpr (kInt8) {
    asm volatile("{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n " ISP_ELECT_PRED
                 " @e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile("{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n " ISP_ELECT_PRED
                 " @e tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  }
}
template <bool kPair>
ISP_D void mma_commit_elect(uint64_t* bar) {
  if constexpr (kPair) {
    asm volatile("{\n .reg .b16 m;\n .reg .pred e;\n mov.b16 m, 3;\n " ISP_ELECT_PRED
                 " @e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], "
                 "m;\n}" ::"r"(smem_u32(bar))
                 : "memory");
  } else {
    asm volatile("{\n .reg .pred e;\n " ISP_ELECT_PRED
                 " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}" ::"r"(
                     smem_u32(bar))
                 : "memory");
  }
}

// 32 TMEM lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
ISP_D void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 TMEM lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
ISP_D void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
ISP_D void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
ISP_D void tmem_ld_wait(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]),
                 "+r"(s[6]), "+r"(s[7]), "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]), "+r"(s[12]),
                 "+r"(s[13]), "+r"(s[14]), "+r"(s[15])
               :
               : "memory");
}
// Wait for outstanding tcgen05.ld and tie the loaded registers to the wait, so
// no use of them can be scheduled before it.
ISP_D void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
ISP_D void tmem_ld_wait(uint32_t (&r)[32], uint32_t (&s)[32]) {
  tmem_ld_wait(r);
  asm volatile(""
               : "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]), "+r"(s[6]), "+r"(s[7]),
                 "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]), "+r"(s[12]), "+r"(s[13]), "+r"(s[14]),
                 "+r"(s[15]), "+r"(s[16]), "+r"(s[17]), "+r"(s[18]), "+r"(s[19]), "+r"(s[20]), "+r"(s[21]),
                 "+r"(s[22]), "+r"(s[23]), "+r"(s[24]), "+r"(s[25]), "+r"(s[26]), "+r"(s[27]), "+r"(s[28]),
                 "+r"(s[29]), "+r"(s[30]), "+r"(s[31]));
}

// ----------------------------------------------------------------------------
// Epilogue helpers
// ----------------------------------------------------------------------------
template <bool kInt8>
ISP_D float acc_value(uint32_t bits) {
  if constexpr (kInt8) return static_cast<float>(static_cast<int32_t>(bits));
  else return __uint_as_float(bits);
}

ISP_D uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
ISP_D uint32_t pack_f16(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// ---- EPI_CONV output staging ----
template <int kN>
ISP_D void st_shared_words(uint8_t* dst, const uint32_t (&w)[kN]) {
  if constexpr (kN == 1) {
    *reinterpret_cast<uint32_t*>(dst) = w[0];
  } else if constexpr (kN == 2) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else {
#pragma unroll
    for (int i = 0; i < kN; i += 4)
      *reinterpret_cast<uint4*>(dst + 4 * i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
  }
}

// One lane's 32 values (columns c * P + r of its phase row q) -> the output box
// [32/P channels][32 rows x P times] (times contiguous): the lane's P values of
// channel c are consecutive times q * P .. q * P + P - 1, written as one vector at
// c * 32P + q * P, so a warp's store covers a contiguous run (no bank conflicts).
template <int kOut, int kP>
ISP_D void stage_conv_box_p(uint8_t* sb, int lane, const float (&v)[32]) {
  constexpr int kEb = kOut == OUT_F32 ? 4 : 2;
#pragma unroll
  for (int c = 0; c < 32 / kP; ++c) {
    uint8_t* dst = sb + (c * 32 * kP + lane * kP) * kEb;
    if constexpr (kEb == 4) {
      uint32_t w[kP];
#pragma unroll
      for (int r = 0; r < kP; ++r) w[r] = __float_as_uint(v[c * kP + r]);
      st_shared_words<kP>(dst, w);
    } else if constexpr (kP == 1) {
      *reinterpret_cast<uint16_t*>(dst) = kOut == OUT_F16 ? __half_as_ushort(__float2half_rn(v[c]))
                                                          : __bfloat16_as_ushort(__float2bfloat16_rn(v[c]));
    } else {
      uint32_t w[kP / 2];
#pragma unroll
      for (int i = 0; i < kP / 2; ++i)
        w[i] = kOut == OUT_F16 ? pack_f16(v[c * kP + 2 * i], v[c * kP + 2 * i + 1])
                               : pack_bf16(v[c * kP + 2 * i], v[c * kP + 2 * i + 1]);
      st_shared_words<kP / 2>(dst, w);
    }
  }
}

template <int kOut>
ISP_D void stage_conv_box(uint8_t* sb, int lane, int phases, const float (&v)[32]) {
  switch (phases) {
    case 1: stage_conv_box_p<kOut, 1>(sb, lane, v); break;
    case 2: stage_conv_box_p<kOut, 2>(sb, lane, v); break;
    case 4: stage_conv_box_p<kOut, 4>(sb, lane, v); break;
    default: stage_conv_box_p<kOut, 8>(sb, lane, v); break;
  }
}

// satfinite saturates +-inf and out-of-range values to +-448 and keeps NaN,
// the same result as the reference's clamp(-448, 448) followed by the cast.
ISP_D uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  return static_cast<uint32_t>(e4m3x2(a, b)) | (static_cast<uint32_t>(e4m3x2(c, d)) << 16);
}

// Write one thread's 128-byte row of the 32 x 128 B staging box (128-byte swizzle).
ISP_D void stage_row(uint8_t* stage, int row, const uint32_t (&w)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 v = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    *reinterpret_cast<uint4*>(stage + row * 128 + ((j ^ (row & 7)) << 4)) = v;
  }
}

ISP_D void load_f32x32(const float* p, float (&v)[32]) {   // 16-byte aligned, uniform across the warp
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p) + j);
    v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
  }
}

ISP_D float silu_mul(float g, float u) {
  const float sig = __fdividef(1.f, 1.f + __expf(-g));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

// Named barrier among the epilogue warps only (id 1).
template <int kEpiThreads>
ISP_D void epilogue_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

ISP_D void lds32(const float* p, float (&v)[32]) {   // uniform address: a broadcast read
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 t = *reinterpret_cast<const float4*>(p + 4 * j);
    v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
  }
}

// Shared layout of the per-tile parameters (512 floats), filled from registers
// fetched one tile ahead so the L2 latency is off the critical path:
//   EPI_SCALE:              [0, BN) w_scale (1 when absent), [256, 256 + BN) bias (0 when absent)
//   EPI_SWIGLU_PAIRED:      [0, 128) s1, [128, 256) s3
//   EPI_SWIGLU_INTERLEAVED: [0, 256) S[2 n0 ...] (gate, up alternating)
//   EPI_NLV:                [64 j, 64 j + 64) AS * WS[jN + n], [256 + 64 j, ...) bias[jN + n]
// Columns at or past N read as 0, so the math needs no column guards.
// For EPI_SCALE with a per-tensor activation scale the staged column scale is
// already sa * w_scale[n] (the product the INT8 reference forms as AS * WS[n]).
template <int kEpi, int kBN, int kEpiThreads>
struct TileParams {
  static_assert(kEpiThreads <= 256, "one or more entries per epilogue thread");
  static constexpr int kPer = 256 / kEpiThreads;
  float a[kPer], b[kPer];   // entries et + kEpiThreads * h of the 256-wide shared arrays

  ISP_D void fetch(const Params& p, int n0, int et) {
#pragma unroll
    for (int h = 0; h < kPer; ++h) {
      const int i = et + kEpiThreads * h;
      float x = 0.f, y = 0.f;
      if constexpr (kEpi == EPI_SCALE || kEpi == EPI_CONV) {
        const int n = n0 + i;
        if (i < kBN && n < p.N) {
          const int c = kEpi == EPI_CONV ? n / p.conv_phases : n;   // EPI_CONV: column -> channel
          x = p.w_scale != nullptr ? __ldg(p.w_scale + c) : 1.f;
          if (p.a_scale_rows == nullptr) x = __fmul_rn(p.a_scale, x);
          y = p.bias != nullptr ? __ldg(p.bias + c) : 0.f;
        }
      } else if constexpr (kEpi == EPI_SWIGLU_PAIRED) {
        const int n = n0 + (i & 127);
        if (n < p.N) x = __ldg((i < 128 ? p.w_scale : p.w_scale2) + n);
      } else if constexpr (kEpi == EPI_NLV) {
        // [64 j, 64 j + 64): projection j's AS * WS and bias of the tile's 64 outputs
        const int n = n0 + (i & 63);
        if (i < kNlvBN && n < p.N) {
          const int64_t c = static_cast<int64_t>(i >> 6) * p.N + n;
          x = __fmul_rn(p.a_scale, __ldg(p.w_scale + c));
          y = __ldg(p.bias + c);
        }
      } else {
        if (n0 + (i >> 1) < p.N) x = __ldg(p.w_scale + 2 * n0 + i);
      }
      a[h] = x;
      b[h] = y;
    }
  }
  ISP_D void store(float* sp, int et) const {
#pragma unroll
    for (int h = 0; h < kPer; ++h) {
      sp[et + kEpiThreads * h] = a[h];
      sp[256 + et + kEpiThreads * h] = b[h];
    }
  }
};

// Issue the TMEM loads of output group g (32 output columns).
template <int kEpi, int kBN>
ISP_D void tmem_load_group(uint32_t t_row, int g, uint32_t (&a)[32], uint32_t (&b)[32]) {
  if constexpr (kEpi == EPI_SCALE || kEpi == EPI_CONV) {
    tmem_ld32(t_row + g * 32, a);
  } else if constexpr (kEpi == EPI_SWIGLU_PAIRED) {
    tmem_ld32(t_row + g * 32, a);                // gate
    tmem_ld32(t_row + kBN / 2 + g * 32, b);      // up
  } else {
    tmem_ld32(t_row + g * 64, a);                // (gate, up) pairs of outputs 32g .. 32g+15
    tmem_ld32(t_row + g * 64 + 32, b);           // outputs 32g+16 .. 32g+31
  }
}

// kRows (per-row activation scale sa):
//   FP8  v = fma(acc * sa, ws[n], bias[n])        (ops/triton/fp8.py:32-33 order)
//   INT8 v = (acc * (sa * ws[n])) + bias[n]
// otherwise the staged scale c[n] already holds sa * ws[n]:
//   FP8  v = fma(acc, c[n], bias[n]);  INT8 v = (acc * c[n]) + bias[n]
// (INT8 keeps separate roundings, as i8_residual_runtime_kernel.py:18-20).
template <bool kInt8, bool kRows>
ISP_D void scale_group(const uint32_t (&r)[32], float sa, const float* ws_s, const float* bs_s, float (&v)[32]) {
  float ws[32], bs[32];
  lds32(ws_s, ws);
  lds32(bs_s, bs);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if constexpr (kInt8) {
      const float c = kRows ? __fmul_rn(sa, ws[j]) : ws[j];
      v[j] = __fadd_rn(__fmul_rn(acc_value<true>(r[j]), c), bs[j]);
    } else {
      const float a = kRows ? __fmul_rn(acc_value<false>(r[j]), sa) : acc_value<false>(r[j]);
      v[j] = __fmaf_rn(a, ws[j], bs[j]);
    }
  }
}

ISP_D void add_residual(const Params& p, int m, int n, float (&v)[32]) {
  const int64_t off = static_cast<int64_t>(m) * p.N + n;
  if (n + 32 <= p.N) {
    if (p.residual_f32) {
      float r[32];
      load_f32x32(static_cast<const float*>(p.residual) + off, r);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], r[j]);
    } else {
      const uint4* q = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.residual) + off);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float f[8];
        bf16x8_to_f32(__ldg(q + h), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * h + j] = __fadd_rn(v[8 * h + j], f[j]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (n + j < p.N) {
        const float r = p.residual_f32 ? __ldg(static_cast<const float*>(p.residual) + off + j)
                                       : __bfloat162float(static_cast<const __nv_bfloat16*>(p.residual)[off + j]);
        v[j] = __fadd_rn(v[j], r);
      }
    }
  }
}

ISP_D void store_dual_e4m3(const Params& p, int m, int n, const float (&v)[32]) {
  uint8_t* o2 = static_cast<uint8_t*>(p.out2) + static_cast<int64_t>(m) * p.N + n;
  uint32_t q[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    q[j] = pack_e4m3x4(__fmul_rn(v[4 * j], p.out2_inv), __fmul_rn(v[4 * j + 1], p.out2_inv),
                       __fmul_rn(v[4 * j + 2], p.out2_inv), __fmul_rn(v[4 * j + 3], p.out2_inv));
  if (n + 32 <= p.N) {
    reinterpret_cast<uint4*>(o2)[0] = make_uint4(q[0], q[1], q[2], q[3]);
    reinterpret_cast<uint4*>(o2)[1] = make_uint4(q[4], q[5], q[6], q[7]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n + j < p.N) o2[j] = static_cast<uint8_t>(q[j >> 2] >> (8 * (j & 3)));
  }
}

// SwiGLU of output group g: h = silu(acc_g * s_g) * (acc_u * s_u), then
// clamp(h * out_inv) (E4M3 codes follow) or its E4M3 round trip * out_scale.
template <int kEpi, int kOut>
ISP_D void swiglu_group(const uint32_t (&a)[32], const uint32_t (&b)[32], const float* sp, int g, float out_inv,
                        float out_scale, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    float gacc, uacc, sg, su;
    if constexpr (kEpi == EPI_SWIGLU_PAIRED) {
      gacc = __uint_as_float(a[j]);
      uacc = __uint_as_float(b[j]);
      sg = sp[g * 32 + j];
      su = sp[128 + g * 32 + j];
    } else {
      const uint32_t(&src)[32] = j < 16 ? a : b;
      const int c = 2 * (j & 15);
      gacc = __uint_as_float(src[c]);
      uacc = __uint_as_float(src[c + 1]);
      sg = sp[g * 64 + 2 * j];
      su = sp[g * 64 + 2 * j + 1];
    }
    v[j] = __fmul_rn(silu_mul(__fmul_rn(gacc, sg), __fmul_rn(uacc, su)), out_inv);
  }
  if constexpr (kOut == OUT_F32) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const uint16_t q2 = e4m3x2(v[j], v[j + 1]);
      v[j] = __fmul_rn(e4m3_to_f32(static_cast<uint8_t>(q2 & 0xFF)), out_scale);
      v[j + 1] = __fmul_rn(e4m3_to_f32(static_cast<uint8_t>(q2 >> 8)), out_scale);
    }
  }
}

// NVFP4 SwiGLU of one 16-output block of one row (one NVFP4 scale block):
//   h = silu(acc_gate * alpha_gate) * (acc_up * alpha_up)
// quantized with the global scale gq:
//   s = e4m3(min(amax(h) / (6 gq), 448)) (an all-zero block takes s = 1),
//   code = e2m1(h / (s gq)), low nibble = even column.
// silu(g) = g/2 * (1 + tanh(g/2)) takes one MUFU op per element, and alpha_up
// is applied once per block: h' = silu(g) * acc_up, amax(h) = amax(h') |alpha_up|,
// h / (s gq) = h' * RN(alpha_up / (s gq)).  The quotient can therefore differ
// from an exactly rounded h / (s gq) by an ulp or two, which moves a code only
// within that distance of a decision point.  A block whose scale rounds to 0
// takes the codes of h / 0: +-6 for h != 0, 0 for h == 0.
// ag_half = alpha_gate / 2; r6 = RN(1 / (6 gq)).  Returns the 8 code bytes
// (low word = columns 0-7) and the scale byte in `sf`.
ISP_D float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

ISP_D uint2 swiglu_nvfp4_block(const uint32_t (&a)[16], const uint32_t (&b)[16], float ag_half, float au, float gq,
                               float six_gq, float r6, uint32_t& sf) {
  float h[16];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float hg = __fmul_rn(__uint_as_float(a[j]), ag_half);
    h[j] = __fmul_rn(__fmaf_rn(hg, tanh_approx(hg), hg), __uint_as_float(b[j]));
    amax = fmaxf(amax, fabsf(h[j]));
  }
  float sb = div_rn_recip(__fmul_rn(amax, fabsf(au)), six_gq, r6);
  if (sb == 0.f) sb = 1.f;
  const uint32_t sc = e4m3x2(fminf(sb, 448.f), 0.f) & 0xFFu;
  sf = sc;
  uint32_t w[2];
  if (sc != 0u) {
    const float r = __fmul_rn(au, __frcp_rn(__fmul_rn(e4m3_to_f32(static_cast<uint8_t>(sc)), gq)));
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t packed = 0;
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float* hp = &h[8 * half + j];
        // fma(h, r, +0) == RN(h r) and turns -0 into +0
        packed |= e2m1x2(__fmaf_rn(hp[0], r, 0.f), __fmaf_rn(hp[1], r, 0.f)) << (4 * j);
      }
      w[half] = packed;
    }
  } else {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t packed = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = __fmul_rn(h[8 * half + j], au);
        packed |= (v > 0.f ? 7u : (v < 0.f ? 15u : 0u)) << (4 * j);
      }
      w[half] = packed;
    }
  }
  return make_uint2(w[0], w[1]);
}

// ----------------------------------------------------------------------------
// Tile schedule
// ----------------------------------------------------------------------------
// Streaming: CTA c takes tiles c, c + grid, ... in M-major order (all CTAs work
// on neighbouring tiles, so A and B re-reads hit L2).  B-stationary: CTA c takes
// a contiguous range of the N-major order, so it crosses at most a few N tiles
// and reloads its resident B tile only there.
template <bool kStat>
struct Schedule {
  int begin, end, step;
  int full;   // streaming with tail_split: units from here on are half-N tiles, two per tile
  // `unit` of `units` workers: the CTA, or the SM pair in the pair schedule
  ISP_D Schedule(const Params& p, int unit, int units) {
    const int total = p.m_tiles * p.n_tiles;
    full = total;
    if constexpr (kStat) {
      begin = static_cast<int>(static_cast<int64_t>(unit) * total / units);
      end = static_cast<int>(static_cast<int64_t>(unit + 1) * total / units);
      step = 1;
    } else {
      begin = unit;
      end = total;
      step = units;
      // The last partial wave (rem tiles) would keep rem CTAs busy while the rest idle;
      // as 2 rem half-N tiles it spreads over twice as many CTAs.
      const int rem = total % units;
      if (p.tail_split && rem > 0 && 2 * rem <= units) {
        full = total - rem;
        end = total + rem;
      }
    }
  }
  // Unit t -> tile (mt, nt); hn = -1 for a whole tile, else the N half (0 / 1) of a split tile.
  ISP_D void coords(const Params& p, int t, int& mt, int& nt, int& hn) const {
    hn = -1;
    if constexpr (!kStat) {
      if (t >= full) {
        hn = (t - full) & 1;
        t = full + ((t - full) >> 1);
      }
    }
    if constexpr (kStat) {
      nt = t / p.m_tiles;
      mt = t - nt * p.m_tiles;
    } else {
      mt = t / p.n_tiles;
      nt = t - mt * p.n_tiles;
    }
  }
};

// ----------------------------------------------------------------------------
// The kernel
// ----------------------------------------------------------------------------
// kBStatK > 0: B-stationary schedule holding kBStatK bytes of K of the B tile
// resident (requires K bytes <= kBStatK).
// kPair: SM-pair schedule (a cluster of two CTAs, tcgen05 cta_group::2): 256 x kBN tiles,
// CTA rank r holds A rows [128 r, 128 r + 128) and B rows [r kBN / 2, (r + 1) kBN / 2) of
// each tile; the leader (rank 0) issues M = 256 MMAs that read both CTAs' shared memory
// and write each CTA's 128 rows into its own TMEM; both CTAs run the epilogue of their
// rows.  The full / bfull / tempty barriers that gate the MMAs live in the leader (TMA
// bytes of both CTAs and both CTAs' epilogue hand-backs are counted there); the leader's
// commits arrive on the empty / bempty / tfull / drain barriers of both CTAs.
template <int kBN, int kStages, int kEpiWarps, int kAB, int kEpi, int kOut, int kBStatK, bool kPair>
__global__ void __launch_bounds__(kernel_threads<kEpiWarps, kAB == AB_FP4>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_b2, const __grid_constant__ CUtensorMap tm_out,
                const __grid_constant__ Params p) {
  constexpr bool kInt8 = kAB == AB_I8;
  constexpr bool kFp4 = kAB == AB_FP4;
  constexpr bool kStat = kBStatK > 0;
  static_assert(!kFp4 || kBN == 128, "NVFP4 tiles are 128 x 128 (one scale chunk per operand and K = 64)");
  static_assert(kOut != OUT_NVFP4 || (kFp4 && kEpi == EPI_SWIGLU_PAIRED), "NVFP4 output is the FP4 SwiGLU epilogue");
  static_assert(kBStatK % kBK == 0, "resident K is whole 128-byte blocks");
  static_assert(kEpi != EPI_NLV || (kBN == kNlvBN && kAB == AB_I8 && kOut == OUT_F32 && kEpiWarps == 8),
                "nonlinear-value tiles: INT8, 3 x 64 columns, FP32 outputs, two epilogue warps per lane quarter");
  static_assert(!kPair || (kEpi == EPI_SCALE && !kFp4 && kBN == 256),
                "SM-pair tiles: 256 x 256 FP8 / INT8 scale GEMMs (B-stationary or streaming)");
  constexpr int kBRows = kPair ? kBN / 2 : kBN;   // B rows in this CTA's shared memory
  constexpr int kTileM = kPair ? 2 * kBM : kBM;   // rows of one tile
  constexpr int kStagingBufs = kPair ? kStagingBufsPair : kStagingBufsOne;
  using L = Smem<kBRows, kStages, kEpiWarps, kFp4, kOut != OUT_NVFP4 && kEpi != EPI_NLV, kBStatK, kStagingBufs>;
  using R = Roles<kEpiWarps>;
  using S = Schedule<kStat>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The 128-byte swizzle patterns assume a 1024-byte aligned base; refuse to run otherwise.
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicExch(&g_device_error, (int)ISP_ERR_ALIGN);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* staging = smem + L::kStagingOffset;
  float* params = reinterpret_cast<float*>(smem + L::kParamOffset);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty_bar = full_bar + kStages;
  // TMEM accumulators: two; B-stationary NVFP4 tiles (one 128-column accumulator per
  // 512 MMA cycles, shorter than the accumulator hand-back round trip) keep three.
  constexpr int kAccs = (kFp4 && kStat) ? 3 : 2;
  uint64_t* tfull_bar = empty_bar + kStages;     // [kAccs]
  uint64_t* tempty_bar = tfull_bar + kAccs;      // [kAccs]
  uint64_t* drain_bar = tempty_bar + kAccs;      // [1]
  uint64_t* bfull_bar = drain_bar + 1;           // [1] resident B landed (B-stationary)
  uint64_t* bempty_bar = bfull_bar + 1;          // [1] every MMA reading the resident B completed
  uint64_t* sf_bar = bempty_bar + 1;            // [kStages] NVFP4: the stage's scales are in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_bar + (kFp4 ? kStages : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // TMEM: two accumulators (columns [0, 2 kBN)); NVFP4 adds its scale columns after
  // them: streaming 32 per stage (A 16, B 16); B-stationary the resident B scales
  // (4 per 64-element K chunk) and 16 A columns per stage.
  // (allocations are powers of two: two 192-column nonlinear-value accumulators take 512)
  constexpr int kTmemCols = (kFp4 || kEpi == EPI_NLV) ? 512 : 2 * kBN;
  // NVFP4 scale columns of a stage's A (streaming: A and B) scales; with three
  // accumulators the stages share four slots, a slot being rewritten only after the
  // MMAs of its previous stage completed (the scale warp waits for that stage's empty
  // barrier).
  constexpr int kSfSlots = kAccs == 3 ? 4 : kStages;
  static_assert(kSfSlots <= kStages, "a slot's previous stage is at most one ring round back");
  constexpr int kSfbResCols = kStat ? (2 * kBStatK / 64) * 4 : 0;
  static_assert(!kFp4 || kAccs * kBN + kSfbResCols + (kStat ? 16 : 32) * kSfSlots <= 512, "TMEM columns");

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < kAccs; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kPair ? 2 * kEpiWarps : kEpiWarps);   // one arrive per epilogue warp
    }
    mbar_init(drain_bar, 1);
    mbar_init(bfull_bar, 1);
    mbar_init(bempty_bar, 1);
    if constexpr (kFp4)
      for (int s = 0; s < kStages; ++s) mbar_init(&sf_bar[s], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    if constexpr (kEpi == EPI_SWIGLU_PAIRED) prefetch_tmap(&tm_b2);
    if constexpr (kOut != OUT_NVFP4) prefetch_tmap(&tm_out);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  // pair: both CTAs' barriers are initialized before either sends a remote arrive or bytes
  if constexpr (kPair) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t rank = kPair ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const S sched(p, kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x),
                kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x));
  // Resident B tile `nt` (B-stationary): the weight rows of one N tile, all of K.
  auto load_resident_b = [&](int nt) {
    uint32_t bytes = static_cast<uint32_t>(p.k_blocks) * L::kBBytes;
    if constexpr (kFp4) bytes += static_cast<uint32_t>(p.k_chunks) * kSfChunk;
    if constexpr (kPair) {
      if (lane == 0 && leader) mbar_expect_tx(bfull_bar, 2 * bytes);      // both halves land on the leader's
    } else {
      if (lane == 0) mbar_expect_tx(bfull_bar, bytes);
    }
    for (int kb = 0; kb < p.k_blocks && lane == 0; ++kb) {
      uint8_t* dst = smem + L::kBResOffset + kb * L::kBBytes;
      if constexpr (kPair) {
        tma_load_2d_pair<true>(dst, &tm_b, map_to_rank(smem_u32(bfull_bar), 0), kb * kBK,
                         nt * kBN + static_cast<int>(rank) * kBRows);
      } else if constexpr (kEpi == EPI_SWIGLU_PAIRED && !kFp4) {
        tma_load_2d(dst, &tm_b, bfull_bar, kb * kBK, nt * (kBN / 2));
        tma_load_2d(dst + (kBN / 2) * kBK, &tm_b2, bfull_bar, kb * kBK, nt * (kBN / 2));
      } else if constexpr (kEpi == EPI_NLV) {
        for (int j = 0; j < 3; ++j)
          tma_load_2d(dst + j * (kBN / 3) * kBK, &tm_b, bfull_bar, kb * kBK, j * p.N + nt * (kBN / 3));
      } else {
        tma_load_2d(dst, &tm_b, bfull_bar, kb * kBK, nt * kBN);
      }
    }
    if constexpr (kFp4)
      if (lane == 0)
        bulk_load(smem + L::kSfbResOffset, p.sfb + static_cast<int64_t>(nt) * p.k_chunks * kSfChunk,
                  static_cast<uint32_t>(p.k_chunks) * kSfChunk, bfull_bar);
  };
  // The prologue above touches no global memory.  The weight does not depend on the
  // preceding kernel: the producer loads the first resident B tile before waiting
  // for it, so that load overlaps the predecessor's tail.  Everything else (A, the
  // epilogue's parameters, residuals and outputs) waits; then the next kernel may
  // start its own prologue.
  int pre_nt = -1;
  if constexpr (kStat) {
    if (warp == 0 && sched.begin < sched.end) {
      int mt0, hn0;
      sched.coords(p, sched.begin, mt0, pre_nt, hn0);
      load_resident_b(pre_nt);
      __syncwarp();
    }
  }
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop (waits converged); lane 0 issues the copies.
    {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_phase[kStages];
      bool armed[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) armed[s] = false, armed_phase[s] = 0;
      bool ok = true;
      int cur_nt = pre_nt;                       // loaded before the dependency wait
      uint32_t nloads = pre_nt >= 0 ? 1u : 0u;   // resident-B loads issued
      for (int t = sched.begin; t < sched.end && ok; t += sched.step) {
        int mt, nt, hn;
        sched.coords(p, t, mt, nt, hn);   // a half-N tile loads the whole tile's A and B
        const int m0 = mt * kTileM + static_cast<int>(rank) * kBM;
        if constexpr (kStat) {
          if (nt != cur_nt) {
            // reload the resident B tile once every MMA reading the previous one completed
            if (nloads > 0 && !wait_warp(bempty_bar, (nloads - 1) & 1u, abort_flag)) { ok = false; break; }
            load_resident_b(nt);
            __syncwarp();
            cur_nt = nt;
            ++nloads;
          }
        }
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_warp(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          armed[stage] = true;
          armed_phase[stage] = phase;
          if (lane == 0) {
            uint8_t* sa = smem + L::a(stage);
            uint32_t bytes = L::kABytes + (kStat ? 0 : L::kBBytes);
            const int nch = kFp4 ? min(4, p.k_chunks - 4 * kb) : 0;   // 64-element scale chunks of this stage
            if constexpr (kFp4) bytes += static_cast<uint32_t>(nch) * kSfChunk * (kStat ? 1 : 2);
            if constexpr (kPair) {
              if (leader) mbar_expect_tx(&full_bar[stage], 2 * bytes);
              tma_load_2d_pair<kStat>(sa, &tm_a, map_to_rank(smem_u32(&full_bar[stage]), 0), kb * kBK, m0);
            } else {
              mbar_expect_tx(&full_bar[stage], bytes);
            }
            if constexpr (kPair) {
            } else if constexpr (kEpi == EPI_CONV) {
              const int b = mt / p.conv_tpb;
              const int j = kb / p.conv_cblocks;
              const int e = p.conv_tab[j];
              const int q0 = (mt - b * p.conv_tpb) * kBM;
              tma_load_3d(sa, &tm_a, &full_bar[stage], ((e & 1023) + kb - j * p.conv_cblocks) * kBK, q0 + (e >> 10), b);
            } else {
              tma_load_2d(sa, &tm_a, &full_bar[stage], kb * kBK, m0);
            }
            if constexpr (kFp4) {
              const int64_t a_off = (static_cast<int64_t>(mt) * p.k_chunks + 4 * kb) * kSfChunk;
              bulk_load(smem + L::sfa(stage), p.sfa + a_off, static_cast<uint32_t>(nch) * kSfChunk, &full_bar[stage]);
            }
            if constexpr (!kStat) {
              uint8_t* sb = smem + L::b(stage);
              if constexpr (kPair) {   // this CTA's half of the stage's B rows, bytes on the leader's barrier
                tma_load_2d_pair<true>(sb, &tm_b, map_to_rank(smem_u32(&full_bar[stage]), 0), kb * kBK,
                                 nt * kBN + static_cast<int>(rank) * kBRows);
              } else if constexpr (kEpi == EPI_SWIGLU_PAIRED && !kFp4) {
                tma_load_2d(sb, &tm_b, &full_bar[stage], kb * kBK, nt * (kBN / 2));
                tma_load_2d(sb + (kBN / 2) * kBK, &tm_b2, &full_bar[stage], kb * kBK, nt * (kBN / 2));
              } else if constexpr (kEpi == EPI_NLV) {
                for (int j = 0; j < 3; ++j)
                  tma_load_2d(sb + j * (kBN / 3) * kBK, &tm_b, &full_bar[stage], kb * kBK, j * p.N + nt * (kBN / 3));
              } else {
                tma_load_2d(sb, &tm_b, &full_bar[stage], kb * kBK, nt * kBN);
              }
              if constexpr (kFp4) {
                const int64_t b_off = (static_cast<int64_t>(nt) * p.k_chunks + 4 * kb) * kSfChunk;
                bulk_load(smem + L::sfb(stage), p.sfb + b_off, static_cast<uint32_t>(nch) * kSfChunk, &full_bar[stage]);
              }
            }
          }
          __syncwarp();
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: every armed stage's last load (and the last resident B) has landed before
      // the CTA exits, also when another role gave up (a copy in flight still lands).
      // (pair: the loads count on the leader's barriers; the peer's warp 1 waits for the
      // leader's final MMA commit instead, which follows every load the MMAs consumed)
      if (!kPair || leader) {
        for (int s = 0; s < kStages; ++s)
          if (armed[s]) wait_warp_drain(&full_bar[s], armed_phase[s]);
        if (kStat && nloads > 0) wait_warp_drain(bfull_bar, (nloads - 1) & 1u);
      }
    }
  } else if (kFp4 && warp == kEpiWarp0 + kEpiWarps) {
    // ------------------------------------------------------------ scale copies (NVFP4)
    // Walks the MMA warp's stage sequence: once a stage has landed, its block scales
    // (A; streaming also B) go to the stage's TMEM scale columns and a commit on
    // sf_bar[stage] signals their completion.  A stage's columns are rewritten only
    // after its next TMA load, i.e. after the MMAs of its previous use completed.
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    bool armed[kStages];
    uint32_t armed_phase[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) armed[s] = false, armed_phase[s] = 0;
    int uses = 0;                                   // stages consumed so far
    int slot = 0;                                   // = uses mod kSfSlots
    for (int t = sched.begin; t < sched.end && ok; t += sched.step) {
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        if (!wait_warp(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
        if (kSfSlots < kStages && uses >= kSfSlots) {
          // the MMAs of the stage that last used this slot have completed
          const int prev = stage >= kSfSlots ? stage - kSfSlots : stage + kStages - kSfSlots;
          const uint32_t prev_phase = stage >= kSfSlots ? phase : phase ^ 1u;
          if (!wait_warp(&empty_bar[prev], prev_phase, abort_flag)) { ok = false; break; }
        }
        ++uses;
        tc_fence_after();
        {
          const int nch = min(4, p.k_chunks - 4 * kb);
          const uint32_t sfa_t =
              tmem_base + static_cast<uint32_t>(kAccs * kBN + kSfbResCols + (kStat ? 16 : 32) * slot);
          const uint32_t sf_s = smem_u32(smem + L::sfa(stage));
          for (int c = 0; c < nch; ++c) {
            tmem_cp_sf_elect(sfa_t + 4 * c, smem_desc_sf(sf_s + c * kSfChunk));
            if constexpr (!kStat)
              tmem_cp_sf_elect(sfa_t + 16 + 4 * c, smem_desc_sf(smem_u32(smem + L::sfb(stage)) + c * kSfChunk));
          }
          mma_commit_elect<false>(&sf_bar[stage]);
        }
        __syncwarp();
        armed[stage] = true;
        armed_phase[stage] = phase;
        if (++slot == kSfSlots) slot = 0;
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
    // Drain: every issued copy has completed before TMEM is released (also on abort).
    for (int s = 0; s < kStages; ++s)
      if (armed[s]) wait_warp_drain(&sf_bar[s], armed_phase[s]);
  } else if (warp == 1 && kPair && !leader) {
    // pair peer: no MMAs here; before the CTA may retire, wait for the leader's final
    // commit (every MMA reading this CTA's shared memory has completed)
    wait_warp_drain(drain_bar, 0);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (waits converged); one elected lane issues tcgen05 ops.
    {
      const uint32_t idesc = instr_desc<kAB, kBN, kTileM>();
      const uint32_t idesc_half = instr_desc<kAB, kBN / 2>();   // half-N tiles of the split tail
      const uint32_t sfb_res_t = tmem_base + static_cast<uint32_t>(kAccs * kBN);   // B-stationary NVFP4
      int stage = 0;
      int sf_slot = 0;                           // NVFP4 scale slot: stages consumed mod kSfSlots
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      int cur_nt = -1;
      uint32_t bphase = 0;
      for (int t = sched.begin; t < sched.end && ok; t += sched.step) {
        int mt, nt, hn;
        sched.coords(p, t, mt, nt, hn);
        (void)mt;
        if constexpr (kStat) {
          if (nt != cur_nt) {
            if (cur_nt >= 0 && lane == 0) {   // arrives when every MMA on the old B completed
              if constexpr (kPair) mma_commit_pair(bempty_bar);
              else mma_commit(bempty_bar);
            }
            __syncwarp();
            if (!wait_warp(bfull_bar, bphase, abort_flag)) break;
            bphase ^= 1u;
            tc_fence_after();
            if constexpr (kFp4) {
              if (lane == 0) {
                const uint32_t src = smem_u32(smem + L::kSfbResOffset);
                for (int c = 0; c < p.k_chunks; ++c) tmem_cp_sf(sfb_res_t + 4 * c, smem_desc_sf(src + c * kSfChunk));
              }
              __syncwarp();
            }
            cur_nt = nt;
          }
        }
        if (!wait_warp(&tempty_bar[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          // NVFP4: sf_bar[stage] completes only after the scale warp has seen this stage's
          // full barrier (the TMA bytes landed) and its copies of the stage's scales have
          // completed, so the MMA warp waits on sf_bar alone (an mbarrier wait costs its
          // warp ~150 cycles even on a completed phase: gated-up 139 -> 133 us).
          if (!kFp4 && !wait_warp(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          if constexpr (kFp4)   // the scale warp's copies of this stage have completed
            if (!wait_warp(&sf_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          {   // the whole warp: operands computed warp-wide, one elected lane issues
            const uint32_t a_addr = smem_u32(smem + L::a(stage));
            const uint32_t b_addr =
                kStat ? smem_u32(smem + L::kBResOffset + kb * L::kBBytes) : smem_u32(smem + L::b(stage));
            if constexpr (kFp4) {
              // One K = 64 MMA per scale chunk; the chunks are in this stage's TMEM
              // scale columns (copied by the scale warp, completion on sf_bar).
              const int nch = min(4, p.k_chunks - 4 * kb);
              const uint32_t sfa_t =
                  tmem_base + static_cast<uint32_t>(kAccs * kBN + kSfbResCols + (kStat ? 16 : 32) * sf_slot);
              for (int kk = 0; kk < nch; ++kk) {
                const uint32_t sfb_t = kStat ? sfb_res_t + 4 * (4 * kb + kk) : sfa_t + 16 + 4 * kk;
                mma_fp4_elect(d_tmem, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), idesc,
                              sfa_t + 4 * kk, sfb_t, (kb | kk) != 0);
              }
            } else {
              // half-N tile: N = kBN / 2 on B rows [hn kBN / 2, (hn + 1) kBN / 2) of the stage
              const uint32_t bh = hn > 0 ? b_addr + static_cast<uint32_t>((kBN / 2) * kBK) : b_addr;
              const uint32_t id = hn >= 0 ? idesc_half : idesc;
#pragma unroll
              for (int kk = 0; kk < kBK / 32; ++kk) {
                mma_issue_elect<kInt8, kPair>(d_tmem, smem_desc_sw128(a_addr + kk * 32),
                                              smem_desc_sw128(bh + kk * 32), id, (kb | kk) != 0);
              }
            }
            mma_commit_elect<kPair>(&empty_bar[stage]);
          }
          __syncwarp();
          issued = true;
          if (++sf_slot == kSfSlots) sf_slot = 0;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_elect<kPair>(&tfull_bar[acc]);
        __syncwarp();
        if (++acc == kAccs) { acc = 0; acc_phase ^= 1u; }
      }
      // Drain: all issued MMAs have completed before TMEM is released (also on abort).
      if (issued) {
        if (lane == 0) {
          if constexpr (kPair) mma_commit_pair(drain_bar);   // also releases the peer's warp 1
          else mma_commit(drain_bar);
        }
        __syncwarp();
        wait_warp_drain(drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - kEpiWarp0;             // 0 .. kEpiWarps-1
    const int et = threadIdx.x - kEpiWarp0 * 32; // 0 .. kEpiThreads-1
    const int quarter = warp & 3;                // TMEM lane quarter this warp may access
    if constexpr (kEpi == EPI_NLV) {
      // 8 warps: TMEM lane quarter x 32-column half of the tile's 64 outputs.  Each
      // thread owns one row: z0, z1, z2 of its 32 outputs, value = tanh(z0) * z1 to
      // row (b, t) of [groups, M / groups, N], gate = z2 to row m of [M, N].
      const int half = ew >> 2;
      const int row_in_tile = quarter * 32 + lane;
      const int64_t steps = p.M / p.nlv_groups;   // T: rows are m = t * groups + b
      int acc = 0;
      uint32_t acc_phase = 0;
      TileParams<kEpi, kBN, R::kEpiThreads> tp;
      if (sched.begin < sched.end) {
        int mt, nt, hn;
        sched.coords(p, sched.begin, mt, nt, hn);
        tp.fetch(p, nt * (kBN / 3), et);
      }
      for (int t = sched.begin; t < sched.end; t += sched.step) {
        int mt, nt, hn;
        sched.coords(p, t, mt, nt, hn);
        epilogue_sync<R::kEpiThreads>();
        tp.store(params, et);
        epilogue_sync<R::kEpiThreads>();
        if (t + sched.step < sched.end) {
          int mt2, nt2, hn2;
          sched.coords(p, t + sched.step, mt2, nt2, hn2);
          tp.fetch(p, nt2 * (kBN / 3), et);
        }
        if (!wait_bounded(&tfull_bar[acc], acc_phase, abort_flag)) break;
        tc_fence_after();
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kBN);
        uint32_t z0[32], z1[32], z2[32];
        tmem_ld32(t_row + half * 32, z0);
        tmem_ld32(t_row + kBN / 3 + half * 32, z1);
        tmem_ld32(t_row + 2 * (kBN / 3) + half * 32, z2);
        tmem_ld_wait(z0, z1);
        asm volatile("" : "+r"(z2[0]), "+r"(z2[1]), "+r"(z2[2]), "+r"(z2[3]), "+r"(z2[4]), "+r"(z2[5]), "+r"(z2[6]),
                     "+r"(z2[7]), "+r"(z2[8]), "+r"(z2[9]), "+r"(z2[10]), "+r"(z2[11]), "+r"(z2[12]), "+r"(z2[13]),
                     "+r"(z2[14]), "+r"(z2[15]), "+r"(z2[16]), "+r"(z2[17]), "+r"(z2[18]), "+r"(z2[19]), "+r"(z2[20]),
                     "+r"(z2[21]), "+r"(z2[22]), "+r"(z2[23]), "+r"(z2[24]), "+r"(z2[25]), "+r"(z2[26]), "+r"(z2[27]),
                     "+r"(z2[28]), "+r"(z2[29]), "+r"(z2[30]), "+r"(z2[31]));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        if (++acc == kAccs) { acc = 0; acc_phase ^= 1u; }
        const int m = mt * kBM + row_in_tile;
        if (m >= p.M) continue;
        const int c0 = half * 32;
        const int n = nt * (kBN / 3) + c0;
        // z = acc * (AS * WS) + bias (separate roundings: int8_nonlinear_value_runtime_kernel.py:26-28)
        float v[32], gz[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float a0 = __fadd_rn(__fmul_rn(acc_value<true>(z0[j]), params[c0 + j]), params[256 + c0 + j]);
          const float a1 = __fadd_rn(__fmul_rn(acc_value<true>(z1[j]), params[64 + c0 + j]), params[320 + c0 + j]);
          gz[j] = __fadd_rn(__fmul_rn(acc_value<true>(z2[j]), params[128 + c0 + j]), params[384 + c0 + j]);
          v[j] = __fmul_rn(tanhf(a0), a1);
        }
        const int64_t b = m % p.nlv_groups;
        const int64_t ts = m / p.nlv_groups;
        float* vrow = static_cast<float*>(p.out) + (b * steps + ts) * p.N + n;
        float* grow = p.nlv_gate + static_cast<int64_t>(m) * p.N + n;
        if (n + 32 <= p.N) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            *reinterpret_cast<float4*>(vrow + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            *reinterpret_cast<float4*>(grow + j) = make_float4(gz[j], gz[j + 1], gz[j + 2], gz[j + 3]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n + j < p.N) {
              vrow[j] = v[j];
              grow[j] = gz[j];
            }
        }
      }
    } else if constexpr (kOut == OUT_NVFP4) {
      // 16 warps: TMEM lane quarter x 16-column block of the tile's 64 outputs;
      // each thread quantizes one NVFP4 block (16 outputs) of its row per tile.
      static_assert(kOut != OUT_NVFP4 || kEpiWarps == 16, "NVFP4 epilogue layout");
      const int blk = ew >> 2;
      const float ag_half = 0.5f * p.a_scale;
      const float six_gq = __fmul_rn(6.f, p.q_scale);
      const float r6 = __frcp_rn(six_gq);
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = sched.begin; t < sched.end; t += sched.step) {
        int mt, nt, hn;
        sched.coords(p, t, mt, nt, hn);   // (never split: the scale epilogue only)
        const int m = mt * kBM + quarter * 32 + lane;
        const int n = nt * (kBN / 2) + 16 * blk;    // first output column of this block
        if (!wait_bounded(&tfull_bar[acc], acc_phase, abort_flag)) break;
        tc_fence_after();
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kBN);
        uint32_t ga[16], ua[16];
        tmem_ld16(t_row + 16 * blk, ga);               // gate columns of this block
        tmem_ld16(t_row + kBN / 2 + 16 * blk, ua);     // up columns
        tmem_ld_wait(ga, ua);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        uint32_t sc;
        const uint2 q = swiglu_nvfp4_block(ga, ua, ag_half, p.alpha_up, p.q_scale, six_gq, r6, sc);
        if (m < p.M) {
          *reinterpret_cast<uint2*>(p.q_codes + static_cast<int64_t>(m) * (p.N / 2) + n / 2) = q;
          p.q_sf[(static_cast<int64_t>(m >> 7) * (p.N / 64) + (n >> 6)) * kSfChunk + (m & 31) * 16 +
                 ((m >> 5) & 3) * 4 + ((n >> 4) & 3)] = static_cast<uint8_t>(sc);
        }
        if (++acc == kAccs) { acc = 0; acc_phase ^= 1u; }
      }
    } else {
      const int half = ew / 4;                     // which share of the columns (8-warp epilogue)
      const int row_in_tile = quarter * 32 + lane;
      uint8_t* stage_base = staging + ew * (kStagingBufs * 32 * 128);
      int sbuf = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      constexpr bool kScaleLike = kEpi == EPI_SCALE || kEpi == EPI_CONV;
      constexpr int kOutCols = kScaleLike ? kBN : kBN / 2;
      constexpr int kChunkCols = 128 / (kOut == OUT_F32 ? 4 : (kOut == OUT_E4M3 ? 1 : 2));
      constexpr int kGroupsPerChunk = kChunkCols / 32;
      constexpr int kGroups = kOutCols / 32 / R::kHalves;   // 32-column groups this warp handles
      static_assert(kGroups % kGroupsPerChunk == 0, "a warp's columns must be whole store boxes");
      const int g0 = half * kGroups;
      constexpr int kWordsPerGroup = 32 / kGroupsPerChunk;
      TileParams<kEpi, kBN, R::kEpiThreads> tp;
      if (sched.begin < sched.end) {
        int mt, nt, hn;
        sched.coords(p, sched.begin, mt, nt, hn);
        tp.fetch(p, nt * kOutCols + (hn > 0 ? kOutCols / 2 : 0), et);
      }
      int staged_n0 = -1;                        // first column of the parameters in shared memory
      for (int t = sched.begin; t < sched.end; t += sched.step) {
        int mt, nt, hn;
        sched.coords(p, t, mt, nt, hn);
        const int m0 = mt * kTileM + static_cast<int>(rank) * kBM;     // this CTA's 128 rows of the tile
        const int n0 = nt * kOutCols + (hn > 0 ? kOutCols / 2 : 0);   // half-N tile: its columns
        // Per-column parameters -> shared memory (zero past column N) only when this
        // tile's columns differ from the staged ones (a B-stationary range keeps one N
        // tile for many consecutive tiles, so the two epilogue barriers are rare); then
        // start fetching those of the next tile with different columns.
        if (n0 != staged_n0) {
          epilogue_sync<R::kEpiThreads>();
          tp.store(params, et);
          epilogue_sync<R::kEpiThreads>();
          staged_n0 = n0;
          for (int t2 = t + sched.step; t2 < sched.end; t2 += sched.step) {
            int mt2, nt2, hn2;
            sched.coords(p, t2, mt2, nt2, hn2);
            const int c2 = nt2 * kOutCols + (hn2 > 0 ? kOutCols / 2 : 0);
            if (c2 != n0) {
              tp.fetch(p, c2, et);
              break;
            }
          }
        }
        if (!wait_bounded(&tfull_bar[acc], acc_phase, abort_flag)) break;
        tc_fence_after();
        if (hn >= 0 && half == 1) {
          // a half-N tile fills accumulator columns [0, kBN / 2) only: nothing for the
          // warps of the upper columns but handing the accumulator back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (kPair) mbar_arrive_cluster(map_to_rank(smem_u32(&tempty_bar[acc]), 0));
            else mbar_arrive(&tempty_bar[acc]);
          }
          if (++acc == kAccs) { acc = 0; acc_phase ^= 1u; }
          continue;
        }
        const int m = m0 + row_in_tile;
        // EPI_CONV: the row is phase row cq of utterance cu (output times cq * P + r)
        const int cu = kEpi == EPI_CONV ? mt / p.conv_tpb : 0;
        const int64_t cq = kEpi == EPI_CONV ? static_cast<int64_t>(mt - cu * p.conv_tpb) * kBM + row_in_tile : 0;
        const bool row_ok = kEpi == EPI_CONV ? cq * p.conv_phases < p.conv_tout : m < p.M;
        float sa = p.a_scale;
        if (p.a_scale_rows != nullptr && row_ok) sa = __ldg(p.a_scale_rows + m);
        if constexpr (kEpi == EPI_CONV)
          if (p.conv_amax != nullptr) sa = conv_dynamic_scale(__ldg(p.conv_amax + cu));
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kBN);

        // Groups stream with a one-group TMEM prefetch; the accumulator goes back to
        // the MMA warp as soon as its last group is in registers.
        uint32_t ca[32], cb[32];
        tmem_load_group<kEpi, kBN>(t_row, g0, ca, cb);
        uint32_t w[32];
#pragma unroll
        for (int g = 0; g < kGroups; ++g) {
          if constexpr (kScaleLike) tmem_ld_wait(ca);
          else tmem_ld_wait(ca, cb);
          uint32_t na[32], nb[32];
          if (g + 1 < kGroups) {
            tmem_load_group<kEpi, kBN>(t_row, g0 + g + 1, na, nb);    // overlaps this group's math
          } else {
            // every column of the accumulator is in registers: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (kPair) mbar_arrive_cluster(map_to_rank(smem_u32(&tempty_bar[acc]), 0));
              else mbar_arrive(&tempty_bar[acc]);
            }
          }
          const int col = (g0 + g) * 32;           // first output column of this group, tile-relative
          const int n = n0 + col;
          float v[32];
          if constexpr (kEpi == EPI_CONV) {
            if (p.conv_amax != nullptr) scale_group<kInt8, true>(ca, sa, params + col, params + 256 + col, v);
            else scale_group<kInt8, false>(ca, sa, params + col, params + 256 + col, v);
            if (p.conv_tma_store) {
              // this warp's 32 rows x 32 columns = 32/P channels x 32P consecutive times,
              // staged channel-major (times contiguous) and stored as one box
              if (lane == 0) bulk_wait_read_all();      // the previous box has left the buffer
              __syncwarp();
              stage_conv_box<kOut>(stage_base, lane, p.conv_phases, v);
              fence_proxy_async_smem();
              __syncwarp();
              const int64_t t_first = (cq - lane) * p.conv_phases;
              if (lane == 0 && t_first < p.conv_tout && n < p.N) {
                tma_store_3d(&tm_out, stage_base, static_cast<int>(t_first), n / p.conv_phases, cu);
                bulk_commit();
              }
            } else if (row_ok) {
              // per-element stores to [B, CO, T_out]: column n + j is channel (n + j) / P at
              // time cq * P + (n + j) % P
              int co = n / p.conv_phases;
              int r = n - co * p.conv_phases;
              const int64_t tq = cq * p.conv_phases;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int64_t t = tq + r;
                if (co < p.conv_co && t < p.conv_tout) {
                  const int64_t off = (static_cast<int64_t>(cu) * p.conv_co + co) * p.conv_tout + t;
                  if constexpr (kOut == OUT_F32) static_cast<float*>(p.out)[off] = v[j];
                  else if constexpr (kOut == OUT_F16) static_cast<__half*>(p.out)[off] = __float2half_rn(v[j]);
                  else static_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(v[j]);
                }
                if (++r == p.conv_phases) { r = 0; ++co; }
              }
            }
            if (g + 1 < kGroups) {
#pragma unroll
              for (int j = 0; j < 32; ++j) ca[j] = na[j];
            }
            continue;
          }
          if constexpr (kEpi == EPI_SCALE) {
            if (p.a_scale_rows != nullptr) scale_group<kInt8, true>(ca, sa, params + col, params + 256 + col, v);
            else scale_group<kInt8, false>(ca, sa, params + col, params + 256 + col, v);
            if (p.residual != nullptr && row_ok) add_residual(p, m, n, v);
            if (p.out2 != nullptr && row_ok) store_dual_e4m3(p, m, n, v);
            if constexpr (kOut == OUT_E4M3) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(v[j], p.out_inv);
            }
          } else {
            swiglu_group<kEpi, kOut>(ca, cb, params, g0 + g, p.out_inv, p.out_scale, v);
          }
          const int wo = (g % kGroupsPerChunk) * kWordsPerGroup;
          if constexpr (kOut == OUT_F32) {
#pragma unroll
            for (int j = 0; j < 32; ++j) w[wo + j] = __float_as_uint(v[j]);
          } else if constexpr (kOut == OUT_BF16) {
#pragma unroll
            for (int j = 0; j < 16; ++j) w[wo + j] = pack_bf16(v[2 * j], v[2 * j + 1]);
          } else if constexpr (kOut == OUT_F16) {
#pragma unroll
            for (int j = 0; j < 16; ++j) w[wo + j] = pack_f16(v[2 * j], v[2 * j + 1]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) w[wo + j] = pack_e4m3x4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
          if (g % kGroupsPerChunk == kGroupsPerChunk - 1) {
            // ---- stage + TMA store of the 32-row x 128-byte box
            const int c0 = col - (kGroupsPerChunk - 1) * 32;
            uint8_t* st = stage_base + sbuf * (32 * 128);
            if (lane == 0) {                       // the store that last used this buffer has read it
              if constexpr (kStagingBufs == 2) bulk_wait_read_le1();
              else bulk_wait_read_all();
            }
            __syncwarp();
            stage_row(st, lane, w);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && m0 + quarter * 32 < p.M) {   // boxes wholly below row M are skipped
              tma_store_2d(&tm_out, st, n0 + c0, m0 + quarter * 32);
              bulk_commit();
            }
            if constexpr (kStagingBufs == 2) sbuf ^= 1;
          }
          if (g + 1 < kGroups) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              ca[j] = na[j];
              cb[j] = nb[j];
            }
          }
        }
        if (++acc == kAccs) { acc = 0; acc_phase ^= 1u; }
      }
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  // pair: neither CTA retires while the other may still arrive on its barriers or
  // (leader's MMAs) read its shared memory
  if constexpr (kPair) cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (kPair)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
  }
}

// Self-test of the bounded-wait unwind path (no data, no global memory but the
// error word): one CTA of three warps, as the GEMM's roles.  Warp 1 holds 32 TMEM
// columns; warp 0 waits, converged, on an mbarrier that nothing arrives on, with a
// limit of limit_ns, then records ISP_ERR_TIMEOUT and raises the abort flag; warp 2
// waits on a second such barrier under the regular 1 s limit and leaves as soon as
// it sees the flag; TMEM is freed once all three are back.  Every wait ends.
__global__ void __launch_bounds__(96, 1) wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" ::"r"(smem_u32(&tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  if (warp == 0) {
    wait_warp(&bars[0], 0, abort_flag, limit_ns);          // expires: records the timeout, raises the flag
  } else if (warp == 2) {
    if (threadIdx.x == 64) wait_bounded(&bars[1], 0, abort_flag);   // returns on the flag
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" ::"r"(tmem_base));
}

}  // namespace gemm
}  // namespace isp
