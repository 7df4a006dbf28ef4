// tl_gemm_tc.cu -- tensor-core GEMM engine: tcgen05 (kind::tf32) with 3xTF32
// split accumulation, TMA-staged tiles, accumulator in TMEM (sm_100a).  (The
// CTA-pair kernel also has a hybrid split, tf32 hi*hi plus the cross terms as
// one bf16 chain, and a specialised-warp kernel an fp16 split; both are
// described with them.)
//
// The three reference primitives (tinylm.c:439-537) in one kernel family:
//   C[I,J] (=|+=) sum_r A(i,r) B(r,j)
// with A K-major (reduction contiguous: mm, mm_bt) or MN-major (mm_atb), and B
// MN-major (mm, mm_atb) or K-major (mm_bt).  tcgen05 reads both majors for tf32,
// so no operand is transposed in memory.
//
// 3xTF32: every fp32 operand x is split into hi = tf32(x) and lo = x - hi
// (exact in fp32), and the tile product is accumulated as lo*hi + hi*lo +
// hi*hi in fp32 in TMEM.  The tensor core reads a tf32 operand by dropping the
// low 13 mantissa bits of the fp32 word, so the landed raw tile *is* hi and
// only lo = x - trunc(x) is written.  The dropped lo*lo term and the
// truncation of lo leave a relative error near 2^-20 per product: fp32-level
// results from the tf32 tensor pipe.
//
// CTA roles (320 threads):
//   warp 0      TMA producer: raw fp32 tiles of A and B -> shared memory stage
//   warp 1      TMEM owner and MMA issuer (one elected thread)
//   warps 2..5  split warpgroup: lo of each landed raw tile into its own
//               buffer (the raw tile is read as hi)
//   warps 6..9  accumulator warpgroup: every CHUNK_KB k-blocks the TMEM
//               accumulator (double buffered) is added into fp32 registers;
//               finally the epilogue (registers -> global, plus an optional
//               addend: C itself to accumulate, or a residual)
// Pipeline per stage: full (TMA bytes landed) -> ready (lo written) ->
// empty (MMAs that read the stage finished, via tcgen05.commit); per TMEM
// buffer: accf (chunk finished) -> acce (chunk drained).
//
// Every mbarrier wait is bounded: on expiry the thread records an error code
// in the context's device error word, raises a CTA-wide abort flag and the CTA
// winds down (the MMA thread still waits, bounded, for its own MMAs; TMEM is
// always released).
//
// Two kernels share these tiles and this protocol: gemm_tc_kernel (one CTA
// per 128 x 128 output tile, cta_group::1) and gemm_tc_pair_kernel (a cluster
// of two CTAs per 256 x 256 tile, cta_group::2), which halves the shared-
// memory bytes the tensor pipe reads per flop -- the limit of the one-CTA
// kernel -- and is the default wherever both output sides exceed 128.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <algorithm>
#include <cudaTypedefs.h>
#include "tl_gemm.cuh"
#include "tl_tc_ptx.cuh"
#include "tl_trace.cuh"

namespace tl {
namespace tc {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int TILE_A = BM * BK * 4;                  // 16 KB
constexpr int TILE_B = BN * BK * 4;                  // 16 KB
constexpr int OFF_AHI = 0, OFF_ALO = TILE_A, OFF_BHI = 2 * TILE_A, OFF_BLO = 2 * TILE_A + TILE_B;
constexpr int STAGE_BYTES = 2 * (TILE_A + TILE_B);   // 64 KB
constexpr int TX_BYTES = TILE_A + TILE_B;            // raw bytes TMA lands per stage
constexpr int NUM_THREADS = 320;
constexpr int CHUNK_KB = 4;                          // k-blocks per TMEM chunk (K = 128)
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr int TMEM_COLS = 2 * BN;                    // two fp32 accumulators, 128 lanes x BN columns

// Instruction descriptor: D f32, A/B tf32, M=128, N=BN, majors as given.
__host__ __device__ constexpr uint32_t make_idesc(bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

struct Params {
  float *C;
  int I, J, R, ldc;
  const float *add;      // nullptr, C (accumulate) or a residual, row stride ldc
  int kb_per_split;      // k-blocks per CTA along grid z (split-K)
  // Pair kernel: the reduction's k-blocks [0, seg_end0) read tmA / tmB,
  // [seg_end0, seg_end1) tmA1 / tmB1 and the rest tmA2 / tmB2 (several
  // products summed into one output; INT_MAX when there is one).
  int seg_end0, seg_end1;
  size_t split_stride;   // floats between the partial outputs of consecutive splits
  // Pair kernel, tail split: pair-tiles [0, full_tiles) in grouped order run
  // whole; each later tile runs as tail_splits CTA pairs of tail_kb k-blocks,
  // pair u after the full tiles writing its part of the tile into the 256 x 256
  // slot u of tail_ws (tail_splits <= 1: no tail split).
  int full_tiles, tail_splits, tail_kb;
  float *tail_ws;
  // Pair kernel, fp16 split: max |x| (float bits) of A and B of each product,
  // [A0, B0, A1, B1, A2, B2].
  const unsigned *amax;
  // Pair kernel: RoPE on the output (heads of 64 columns; row i at sequence
  // position i % rope_T), table [T][32]; nullptr: none.
  const float *rope_cos, *rope_sin;
  int rope_T;
  int *err;
};

// One thread's output row of BN accumulators, `valid` of them inside the
// matrix.  The addend (nullptr, the output itself, or a residual) is read 32
// columns at a time before those columns are stored: with each load followed
// by its store, a possibly aliasing store orders every load behind the
// previous one, and the row takes 32 memory round trips instead of 4.
// (An L2 prefetch of the addend rows from the producer thread measured
// slower.)
__device__ __forceinline__ void store_row(float *dst, const float *addp, float (&acc)[BN], int valid) {
  if (valid >= BN) {
    // In quarters of 32 columns: four round trips, and no registers beyond
    // the accumulators' held for the loads in flight (wider groups spill).
#pragma unroll
    for (int e0 = 0; e0 < BN; e0 += 32) {
      if (addp) {
#pragma unroll
        for (int e = e0; e < e0 + 32; e += 4) {
          const float4 old = *reinterpret_cast<const float4 *>(addp + e);
          acc[e] = old.x + acc[e]; acc[e + 1] = old.y + acc[e + 1];
          acc[e + 2] = old.z + acc[e + 2]; acc[e + 3] = old.w + acc[e + 3];
        }
      }
#pragma unroll
      for (int e = e0; e < e0 + 32; e += 4)
        *reinterpret_cast<float4 *>(dst + e) = make_float4(acc[e], acc[e + 1], acc[e + 2], acc[e + 3]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < BN; e++)
      if (e < valid) dst[e] = addp ? addp[e] + acc[e] : acc[e];
  }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  // bars: full[S], ready[S], empty[S], accf[2] (chunk in TMEM buffer b is
  // complete), acce[2] (TMEM buffer b drained into registers)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * STAGES + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i0 = blockIdx.y * BM, j0 = blockIdx.x * BN;
  // Split-K: CTA z reduces k-blocks [kb0, kb0 + nk) and writes its own
  // output slice (a partial when the grid has more than one z).
  const int nk_all = (p.R + BK - 1) / BK;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int nk = max(0, min(nk_all - kb0, p.kb_per_split));
  const int nchunks = (nk + CHUNK_KB - 1) / CHUNK_KB;
  float *const Cout = p.C + (size_t)blockIdx.z * p.split_stride;
  const uint32_t smem_base = smem_u32(smem);
  auto bar_full = [&](int s) { return smem_u32(&bars[s]); };
  auto bar_ready = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto bar_empty = [&](int s) { return smem_u32(&bars[2 * STAGES + s]); };
  auto bar_accf = [&](int b) { return smem_u32(&bars[3 * STAGES + b]); };
  auto bar_acce = [&](int b) { return smem_u32(&bars[3 * STAGES + 2 + b]); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_ready(s), 4);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(bar_accf(b), 1);
      mbar_init(bar_acce(b), 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % STAGES, u = kb / STAGES;
        if (u > 0 && !mbar_wait(bar_empty(s), (u - 1) & 1, abort_flag, p.err, 1)) break;
        issued = kb + 1;
        const uint32_t st = smem_base + s * STAGE_BYTES;
        mbar_arrive_expect_tx(bar_full(s), TX_BYTES);
        const int k0 = (kb0 + kb) * BK;
        if (A_MN) {
#pragma unroll
          for (int b = 0; b < BM / 32; b++) tma_load_2d(st + OFF_AHI + b * 4096, &tmA, bar_full(s), i0 + 32 * b, k0);
        } else {
          tma_load_2d(st + OFF_AHI, &tmA, bar_full(s), k0, i0);
        }
        if (B_MN) {
#pragma unroll
          for (int b = 0; b < BN / 32; b++) tma_load_2d(st + OFF_BHI + b * 4096, &tmB, bar_full(s), j0 + 32 * b, k0);
        } else {
          tma_load_2d(st + OFF_BHI, &tmB, bar_full(s), k0, j0);
        }
      }
      // No copy may still be landing when the CTA exits: wait (bounded) for
      // the last load issued into each stage.  On the normal path these have
      // all been consumed already and the waits return at once.
      for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; kb++) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar_full(kb % STAGES), (kb / STAGES) & 1)) {
          if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicExch(p.err, 6); break; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(A_MN, B_MN);
      int chunk = 0, kin = 0, last_committed = -1;
      bool ok = true;
      for (int kb = 0; kb < nk && ok; kb++) {
        const int s = kb % STAGES, u = kb / STAGES;
        const int b = chunk & 1;
        // A TMEM buffer is reused two chunks later, once it has been drained.
        if (kin == 0 && chunk >= 2 && !mbar_wait(bar_acce(b), ((chunk >> 1) - 1) & 1, abort_flag, p.err, 7)) break;
        if (!mbar_wait(bar_ready(s), u & 1, abort_flag, p.err, 2)) break;
        tc_fence_after();
        const uint32_t st = smem_base + s * STAGE_BYTES;
        const uint32_t d = tmem + b * BN;
#pragma unroll
        for (int kk = 0; kk < BK / 8; kk++) {
          // K-major: advance 32 bytes inside the swizzle atom; MN-major: eight
          // K rows (1 KB) per tf32 MMA-K step.  MN-major atoms along M/N sit
          // 4 KB apart (one TMA box of 32 x 32 floats).
          const uint32_t a_off = A_MN ? kk * 1024 : kk * 32;
          const uint32_t b_off = B_MN ? kk * 1024 : kk * 32;
          constexpr uint32_t a_lbo = A_MN ? 4096 : 16, b_lbo = B_MN ? 4096 : 16;
          constexpr uint32_t a_sbo = A_MN ? 512 : 1024, b_sbo = B_MN ? 512 : 1024;
          constexpr uint32_t a_lay = A_MN ? LAYOUT_SW128_BASE32B : LAYOUT_SW128;
          constexpr uint32_t b_lay = B_MN ? LAYOUT_SW128_BASE32B : LAYOUT_SW128;
          const uint64_t a_hi = smem_desc(st + OFF_AHI + a_off, a_lbo, a_sbo, a_lay);
          const uint64_t a_lo = smem_desc(st + OFF_ALO + a_off, a_lbo, a_sbo, a_lay);
          const uint64_t b_hi = smem_desc(st + OFF_BHI + b_off, b_lbo, b_sbo, b_lay);
          const uint64_t b_lo = smem_desc(st + OFF_BLO + b_off, b_lbo, b_sbo, b_lay);
          tc_mma(d, a_lo, b_hi, idesc, (kin > 0 || kk > 0) ? 1u : 0u);
          tc_mma(d, a_hi, b_lo, idesc, 1);
          tc_mma(d, a_hi, b_hi, idesc, 1);
        }
        tc_commit(bar_empty(s));
        if (++kin == CHUNK_KB || kb == nk - 1) {
          tc_commit(bar_accf(b));
          last_committed = chunk;
          chunk++;
          kin = 0;
        }
      }
      // Always leave with this thread's MMAs finished, so TMEM is idle before
      // it is released (also on the abort path).
      if (kin > 0 || last_committed < chunk - 1 || last_committed < 0) {
        tc_commit(bar_accf(chunk & 1));
        last_committed = chunk;
      }
      const int b = last_committed & 1;
      const long long t0 = clock64();
      while (!mbar_try_wait(bar_accf(b), (last_committed >> 1) & 1)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) { *abort_flag = 1; atomicExch(p.err, 3); break; }
      }
    }
  } else if (warp < 6) {
    // ---------------------------------------------------- split warpgroup
    const int t = threadIdx.x - 64;  // 0..127
    for (int kb = 0; kb < nk; kb++) {
      const int s = kb % STAGES, u = kb / STAGES;
      if (!mbar_wait(bar_full(s), u & 1, abort_flag, p.err, 4)) break;
      uint8_t *st = smem + s * STAGE_BYTES;
      // A tile then B tile: 2 x 1024 float4 of raw data, 16 per thread.
#pragma unroll 4
      for (int e = 0; e < 16; e++) {
        const int idx = e * 128 + t;                    // 0..2047
        const int off = idx < 1024 ? OFF_AHI + idx * 16 : OFF_BHI + (idx - 1024) * 16;
        float4 *src = reinterpret_cast<float4 *>(st + off);
        float4 *dlo = reinterpret_cast<float4 *>(st + off + (idx < 1024 ? TILE_A : TILE_B));
        const float4 x = *src;
        float4 lo;
        lo.x = x.x - tf32_trunc(x.x); lo.y = x.y - tf32_trunc(x.y);
        lo.z = x.z - tf32_trunc(x.z); lo.w = x.w - tf32_trunc(x.w);
        *dlo = lo;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_ready(s));
    }
  } else {
    // ---------------------------------- fp32 accumulation + epilogue warps
    // The tensor pipe adds into TMEM with truncation, so a long reduction
    // kept there loses bits in proportion to its length.  Each chunk of
    // CHUNK_KB k-blocks is therefore drained into fp32 registers and summed
    // with round-to-nearest adds here.
    const int q = warp & 3;
    float acc[BN];
#pragma unroll
    for (int e = 0; e < BN; e++) acc[e] = 0.0f;
    bool ok = true;
    for (int c = 0; c < nchunks; c++) {
      const int b = c & 1;
      if (!mbar_wait(bar_accf(b), (c >> 1) & 1, abort_flag, p.err, 5)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < BN / 32; cc++) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * BN + cc * 32;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
              "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
              "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int e = 0; e < 32; e++) acc[cc * 32 + e] += __uint_as_float(v[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acce(b));
    }
    if (ok) {
      const int row = i0 + q * 32 + lane;
      if (row < p.I) {
        float *dst = Cout + (size_t)row * p.ldc + j0;
        const float *addp = p.add ? p.add + (size_t)row * p.ldc + j0 : nullptr;
        store_row(dst, addp, acc, p.J - j0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------- CTA-pair (2-SM) tensor-core kernel
// A cluster of two CTAs on an SM pair computes one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256).  Each CTA stages only its own
// 128 rows of A and its own 128 columns of B, so per SM the tensor pipe reads
// 8 KB of shared memory per 128-cycle MMA instead of 8 KB per 64 cycles in the
// one-CTA kernel, and L2 serves half the operand bytes per flop.  Tiles in
// shared memory have the one-CTA kernel's shapes and layouts.
//
// Shared memory holds two rings: RAW_STAGES slots of raw tiles (what TMA
// lands; read by the MMA as hi) and LO_STAGES slots of lo tiles (written by
// the split warps).  The raw ring is the deeper one, so loads run up to
// RAW_STAGES k-blocks ahead of the tensor pipe and hide DRAM latency.
//
// Roles: warp 0 loads this CTA's A and B halves (TMA into its own shared
// memory, no multicast); warp 1 of the leader CTA (rank 0) issues the MMAs of
// the pair; warps 2-9 of both CTAs write the lo parts of the landed tiles and
// drain finished TMEM chunks into fp32 registers.  Every split warp of both
// CTAs signals the leader's `ready` barrier once per k-block and its `acce`
// barrier once per chunk, through cluster addresses; the leader's commits
// arrive on the `rempty`/`lempty`/`accf` barriers of both CTAs.
//
// Output tiles are visited in groups of PAIR_GROUP_M pair-rows, so the pairs
// resident at one time share rows of A and columns of B in L2.
constexpr int PM = 2 * BM, PN = 2 * BN;                 // 256 x 256 per pair
#ifndef TL_PAIR_RAW_STAGES
#define TL_PAIR_RAW_STAGES 4
#endif
#ifndef TL_PAIR_LO_STAGES
#define TL_PAIR_LO_STAGES 3
#endif
#ifndef TL_PAIR_GROUP_M
#define TL_PAIR_GROUP_M 4
#endif
constexpr int RAW_STAGES = TL_PAIR_RAW_STAGES, LO_STAGES = TL_PAIR_LO_STAGES;
constexpr int RAW_BYTES = TILE_A + TILE_B;              // 32 KB: A rows, then this CTA's B half
constexpr int PAIR_SMEM_BYTES = (RAW_STAGES + LO_STAGES) * RAW_BYTES + 1024 /*align*/ + 256 /*barriers*/;
#ifndef TL_PAIR_CHUNK_KB
#define TL_PAIR_CHUNK_KB 8
#endif
constexpr int PAIR_CHUNK_KB = TL_PAIR_CHUNK_KB;         // k-blocks per TMEM chunk before promotion
constexpr int PAIR_TMEM_COLS = 2 * PN;                  // two 256-column accumulators
constexpr int PAIR_SIGNALLERS = 2 * 8;                  // split/drain warps in the pair
constexpr int PAIR_DRAIN_LAG = 2;                       // k-blocks split ahead of a forced drain
constexpr int PAIR_GROUP_M = TL_PAIR_GROUP_M;           // pair-rows per tile group
static_assert(PAIR_SMEM_BYTES <= 232448, "pair kernel exceeds the opt-in shared memory per block");

// Grouped order of the pair kernel's output tiles: pair-tile L (launch order)
// -> tile row pm (256 rows) and tile column tn (256 columns), PAIR_GROUP_M
// tile rows at a time, so pairs resident together share rows of A and
// columns of B in L2.
__host__ __device__ inline void pair_tile(int L, int I, int J, int *pm, int *tn) {
  const int npm = (I + PM - 1) / PM, ntn = (J + PN - 1) / PN;
  const int group = L / (PAIR_GROUP_M * ntn), first_pm = group * PAIR_GROUP_M;
  const int gsz = min(npm - first_pm, PAIR_GROUP_M);
  const int in_group = L - group * PAIR_GROUP_M * ntn;
  *pm = first_pm + in_group % gsz;
  *tn = in_group / gsz;
}

__host__ __device__ constexpr uint32_t make_idesc_pair(bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(PN >> 3) << 17) | ((uint32_t)(PM >> 4) << 24);
}

// The fp16 split (engine 4, gemm_tc_pair_f16ws_kernel further down): instead
// of tf32 hi/lo, each operand is scaled by a power of two (so its largest |x|
// lies in [2^14, 2^15)) and split into fp16 hi = x with its low 13
// significand bits cleared (exact in fp16) and lo = rn(x - hi): 11 + 11
// significand bits, the accuracy of the tf32 pair, and fp16 MMAs (kind::f16,
// K = 16) run at twice the tf32 rate.  The converter warps write both parts
// into the lo ring, which then holds the MMA operands (the hybrid split uses
// the same layouts for its bf16 halves): a K-major tile as 128-byte rows
// [hi 32 | lo 32], an MN-major tile as an hi plane and a lo plane (64 MN
// elements per 128-byte row, 8-row groups 1 KB apart, 64-element MN blocks
// 4 KB apart); the raw slot is free once converted.  The epilogue multiplies by the inverse of the product
// scale (exact).  Products summed into one output share one product scale.
__host__ __device__ constexpr uint32_t make_idesc_pair_f16(bool a_mn, bool b_mn) {
  return (1u << 4) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(PN >> 3) << 17) |
         ((uint32_t)(PM >> 4) << 24);
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ uint32_t b2_bits(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t *>(&h); }
// Binary exponent of a max |x| (float bits), limited to +-100 (0 for zero;
// non-finite and subnormal maxima land on the limits).
__device__ __forceinline__ int amax_exp(unsigned bits) {
  return bits == 0 ? 0 : max(-100, min(100, (int)((bits & 0x7fffffffu) >> 23) - 127));
}
__device__ __forceinline__ float exp2i(int k) { return __uint_as_float((uint32_t)(k + 127) << 23); }

// The hybrid split (HYB): hi*hi stays one tf32 product on the raw tile (the
// MMA reads the fp32 values and uses their tf32 part), and the two cross
// terms become one bf16 chain over K-concatenated operands, A as
// [bf16(hi) | bf16(lo)] and B as [bf16(lo) | bf16(hi)] along K:
// sum_k hi_a lo_b + lo_a hi_b.  bf16 keeps fp32's exponent range, so no scale
// is needed; the rounding of hi and lo to bf16 costs at most 2^-18 |a||b| per
// cross term (the tf32 split's lo*hi terms: 2^-20 each).  Per k-block four
// tf32 MMAs and four bf16 MMAs (K = 16) replace twelve tf32 MMAs; the split
// warps write the bf16 halves into the lo ring in the fp16 split's operand
// layouts below, and the raw slot stays until the tf32 products are done.
template <bool A_MN, bool B_MN, bool HYB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                    const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *raw_ring = smem, *lo_ring = smem + RAW_STAGES * RAW_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(lo_ring + LO_STAGES * RAW_BYTES);
  // bars: full[R] (this CTA's raw slot landed), rempty[R] (pair MMAs done
  // with raw slot), ready[L] (both CTAs' lo slot written; leader's copy
  // used), lempty[L] (pair MMAs done with lo slot), accf[2] (chunk in TMEM
  // buffer b complete), acce[2] (buffer b drained; leader's copy used)
  constexpr int NBARS = 2 * RAW_STAGES + 2 * LO_STAGES + 4;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  // The pair's tile and k-block range: grid z splits every tile's reduction
  // (split-K), or the pairs after the full tiles each take a part of a tail
  // tile.
  int L = blockIdx.x >> 1;
  int kb0 = blockIdx.z * p.kb_per_split, kb_len = p.kb_per_split;
  int tail_slot = -1;
  if (p.tail_splits > 1 && L >= p.full_tiles) {
    const int u = L - p.full_tiles;
    L = p.full_tiles + u / p.tail_splits;
    kb0 = (u % p.tail_splits) * p.tail_kb;
    kb_len = p.tail_kb;
    tail_slot = u;
  }
  int pm, tn;
  pair_tile(L, p.I, p.J, &pm, &tn);
  const int i0 = (2 * pm + (int)rank) * BM;    // this CTA's 128 output rows
  const int j0 = tn * PN;                      // the pair's 256 output columns
  const int jb = j0 + (int)rank * BN;          // this CTA's 128 columns of B
  const int nk_all = (p.R + BK - 1) / BK;
  const int nk = max(0, min(nk_all - kb0, kb_len));
  const int nchunks = (nk + PAIR_CHUNK_KB - 1) / PAIR_CHUNK_KB;
  float *const Cout = p.C + (size_t)blockIdx.z * p.split_stride;
  const uint32_t raw_base = smem_u32(raw_ring), lo_base = smem_u32(lo_ring);
  auto bar_full = [&](int s) { return smem_u32(&bars[s]); };
  auto bar_rempty = [&](int s) { return smem_u32(&bars[RAW_STAGES + s]); };
  auto bar_ready = [&](int s) { return smem_u32(&bars[2 * RAW_STAGES + s]); };
  auto bar_lempty = [&](int s) { return smem_u32(&bars[2 * RAW_STAGES + LO_STAGES + s]); };
  auto bar_accf = [&](int b) { return smem_u32(&bars[2 * RAW_STAGES + 2 * LO_STAGES + b]); };
  auto bar_acce = [&](int b) { return smem_u32(&bars[2 * RAW_STAGES + 2 * LO_STAGES + 2 + b]); };
  const uint32_t peer_flag = cluster_map(smem_u32((const void *)abort_flag), rank ^ 1u);

  if (threadIdx.x == 0) {
    for (int s = 0; s < RAW_STAGES; s++) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_rempty(s), 1);   // the pair's MMAs
    }
    for (int s = 0; s < LO_STAGES; s++) {
      mbar_init(bar_ready(s), PAIR_SIGNALLERS);
      mbar_init(bar_lempty(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(bar_accf(b), 1);
      mbar_init(bar_acce(b), PAIR_SIGNALLERS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(PAIR_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  // Both CTAs' barriers are initialised and TMEM allocated before any signal
  // crosses the pair.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % RAW_STAGES, u = kb / RAW_STAGES;
        if (u > 0 && !mbar_wait_pair(bar_rempty(s), (u - 1) & 1, abort_flag, peer_flag, p.err, 1)) break;
        issued = kb + 1;
        const uint32_t st = raw_base + s * RAW_BYTES;
        mbar_arrive_expect_tx(bar_full(s), TX_BYTES);
        // The product this k-block belongs to, and its k offset there.
        int kg = kb0 + kb;
        const CUtensorMap *ta = &tmA, *tb = &tmB;
        if (kg >= p.seg_end1) { ta = &tmA2; tb = &tmB2; kg -= p.seg_end1; }
        else if (kg >= p.seg_end0) { ta = &tmA1; tb = &tmB1; kg -= p.seg_end0; }
        const int k0 = kg * BK;
        if (A_MN) {
#pragma unroll
          for (int b = 0; b < BM / 32; b++) tma_load_2d(st + b * 4096, ta, bar_full(s), i0 + 32 * b, k0);
        } else {
          tma_load_2d(st, ta, bar_full(s), k0, i0);
        }
        if (B_MN) {
#pragma unroll
          for (int b = 0; b < BN / 32; b++) tma_load_2d(st + TILE_A + b * 4096, tb, bar_full(s), jb + 32 * b, k0);
        } else {
          tma_load_2d(st + TILE_A, tb, bar_full(s), k0, jb);
        }
      }
      // No copy may still be landing when the CTA exits.
      for (int kb = issued > RAW_STAGES ? issued - RAW_STAGES : 0; kb < issued; kb++) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar_full(kb % RAW_STAGES), (kb / RAW_STAGES) & 1)) {
          if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicExch(p.err, 6); break; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (leader CTA only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_pair(A_MN, B_MN);
      int chunk = 0, kin = 0, last_committed = -1;
      for (int kb = 0; kb < nk; kb++) {
        const int rs = kb % RAW_STAGES, ls = kb % LO_STAGES;
        const int b = chunk & 1;
        if (kin == 0 && chunk >= 2 &&
            !mbar_wait_pair(bar_acce(b), ((chunk >> 1) - 1) & 1, abort_flag, peer_flag, p.err, 7))
          break;
        if (!mbar_wait_pair(bar_ready(ls), (kb / LO_STAGES) & 1, abort_flag, peer_flag, p.err, 2)) break;
        tc_fence_after();
        const uint32_t hi = raw_base + rs * RAW_BYTES, lo = lo_base + ls * RAW_BYTES;
        const uint32_t d = tmem + b * PN;
        if constexpr (HYB) {
          // tf32 hi*hi on the raw tile, then the cross terms: K-major operands
          // keep [hi | lo] in the two halves of each 128-byte row, MN-major
          // ones in two planes 8 KB apart (2 KB per K = 16 step).
          constexpr uint32_t idesc32 = make_idesc_pair(A_MN, B_MN);
          constexpr uint32_t idescbf = make_idesc_pair_f16(A_MN, B_MN) | (1u << 7) | (1u << 10);   // bf16
#pragma unroll
          for (int kk = 0; kk < BK / 8; kk++) {
            const uint32_t a_off = A_MN ? kk * 1024 : kk * 32;
            const uint32_t b_off = (B_MN ? kk * 1024 : kk * 32) + TILE_A;
            constexpr uint32_t a_lbo = A_MN ? 4096 : 16, b_lbo = B_MN ? 4096 : 16;
            constexpr uint32_t a_sbo = A_MN ? 512 : 1024, b_sbo = B_MN ? 512 : 1024;
            constexpr uint32_t a_lay = A_MN ? LAYOUT_SW128_BASE32B : LAYOUT_SW128;
            constexpr uint32_t b_lay = B_MN ? LAYOUT_SW128_BASE32B : LAYOUT_SW128;
            tc_mma_pair(d, smem_desc(hi + a_off, a_lbo, a_sbo, a_lay), smem_desc(hi + b_off, b_lbo, b_sbo, b_lay),
                        idesc32, (kin > 0 || kk > 0) ? 1u : 0u);
          }
#pragma unroll
          for (int kc = 0; kc < 4; kc++) {
            const int pl = kc >> 1, kk = kc & 1;   // half (plane) of the concatenated K, step in it
            uint64_t op[2];
#pragma unroll
            for (int w = 0; w < 2; w++) {
              const bool mn = w ? B_MN : A_MN;
              const uint32_t t0 = lo + (w ? TILE_A : 0);
              op[w] = mn ? smem_desc(t0 + pl * 8192 + kk * 2048, 4096, 1024, LAYOUT_SW128)
                         : smem_desc(t0 + pl * 64 + kk * 32, 16, 1024, LAYOUT_SW128);
            }
            tc_mma_pair_f16(d, op[0], op[1], idescbf, 1);
          }
          tc_commit_pair(bar_lempty(ls));
          tc_commit_pair(bar_rempty(rs));
        } else {
#pragma unroll
        for (int kk = 0; kk < BK / 8; kk++) {
          const uint32_t a_off = A_MN ? kk * 1024 : kk * 32;
          const uint32_t b_off = (B_MN ? kk * 1024 : kk * 32) + TILE_A;
          constexpr uint32_t a_lbo = A_MN ? 4096 : 16, b_lbo = B_MN ? 4096 : 16;
          constexpr uint32_t a_sbo = A_MN ? 512 : 1024, b_sbo = B_MN ? 512 : 1024;
          constexpr uint32_t a_lay = A_MN ? LAYOUT_SW128_BASE32B : LAYOUT_SW128;
          constexpr uint32_t b_lay = B_MN ? LAYOUT_SW128_BASE32B : LAYOUT_SW128;
          const uint64_t a_hi = smem_desc(hi + a_off, a_lbo, a_sbo, a_lay);
          const uint64_t a_lo = smem_desc(lo + a_off, a_lbo, a_sbo, a_lay);
          const uint64_t b_hi = smem_desc(hi + b_off, b_lbo, b_sbo, b_lay);
          const uint64_t b_lo = smem_desc(lo + b_off, b_lbo, b_sbo, b_lay);
          tc_mma_pair(d, a_lo, b_hi, idesc, (kin > 0 || kk > 0) ? 1u : 0u);
          tc_mma_pair(d, a_hi, b_lo, idesc, 1);
          tc_mma_pair(d, a_hi, b_hi, idesc, 1);
        }
        tc_commit_pair(bar_lempty(ls));
        tc_commit_pair(bar_rempty(rs));
        }
        if (++kin == PAIR_CHUNK_KB || kb == nk - 1) {
          tc_commit_pair(bar_accf(b));
          last_committed = chunk;
          chunk++;
          kin = 0;
        }
      }
      // Leave with the pair's MMAs finished (also on the abort path), so TMEM
      // is idle before it is released.
      if (kin > 0 || last_committed < chunk - 1 || last_committed < 0) {
        tc_commit_pair(bar_accf(chunk & 1));
        last_committed = chunk;
      }
      const int b = last_committed & 1;
      const long long t0 = clock64();
      while (!mbar_try_wait(bar_accf(b), (last_committed >> 1) & 1)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) { pair_abort(abort_flag, peer_flag, p.err, 3); break; }
      }
    }
  } else {
    // ------------------------------ split + fp32 accumulation (warps 2..9)
    // Warp w reads TMEM lanes 32*(w%4).. (its sub-partition) and accumulates
    // columns [128*h, 128*h + 128) of this CTA's 256, h = (w-2)/4.  Chunk c is
    // drained once all its k-blocks are split and its commit has landed,
    // polled between k-blocks and forced PAIR_DRAIN_LAG k-blocks later.
    const int t = threadIdx.x - 64;  // 0..255
    const int q = warp & 3, h = (warp - 2) >> 2;
    float acc[BN];
#pragma unroll
    for (int e = 0; e < BN; e++) acc[e] = 0.0f;
    bool ok = true;
    int kb = 0, c = 0;
    while (kb < nk || c < nchunks) {
      bool drain = false;
      if (c < nchunks) {
        const int c_end = min((c + 1) * PAIR_CHUNK_KB, nk);
        if (kb >= nk || kb >= c_end + PAIR_DRAIN_LAG) {
          drain = true;
        } else if (kb >= c_end) {
          const uint32_t done = lane == 0 ? (mbar_test_cl(bar_accf(c & 1), (c >> 1) & 1) ? 1u : 0u) : 0u;
          drain = __shfl_sync(0xffffffffu, done, 0) != 0;
        }
      }
      if (drain) {
        const int b = c & 1;
        // The whole warp leaves together: tcgen05.ld below is warp-collective.
        const bool landed = mbar_wait_pair(bar_accf(b), (c >> 1) & 1, abort_flag, peer_flag, p.err, 5);
        if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < BN / 32; cc++) {
          uint32_t v[32];
          const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * PN + h * BN + cc * 32;
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
              "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
              : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
              : "r"(taddr));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int e = 0; e < 32; e++) acc[cc * 32 + e] += __uint_as_float(v[e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(cluster_map(bar_acce(b), 0));
        c++;
      } else {
        const int rs = kb % RAW_STAGES, ls = kb % LO_STAGES;
        bool landed = mbar_wait_pair(bar_full(rs), (kb / RAW_STAGES) & 1, abort_flag, peer_flag, p.err, 4);
        if (landed && kb >= LO_STAGES)
          landed = mbar_wait_pair(bar_lempty(ls), ((kb / LO_STAGES) - 1) & 1, abort_flag, peer_flag, p.err, 8);
        if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
        const uint8_t *src = raw_ring + rs * RAW_BYTES;
        uint8_t *dst = lo_ring + ls * RAW_BYTES;
        if constexpr (HYB) {
          // Warps 2-5 convert the A tile, 6-9 this CTA's B half: one raw
          // 128-byte row (32 values) per thread, written as 16-byte chunks.
          const bool is_a = t < 128, mn = is_a ? A_MN : B_MN;
          const int tt = t & 127;
          const uint8_t *sb = src + (is_a ? 0 : TILE_A);
          uint8_t *db = dst + (is_a ? 0 : TILE_A);
          // Raw row and its swizzle: K-major row r = tt (chunk c at c ^ (r % 8));
          // MN-major box tt / 32, K row k = tt % 32 (chunk c at c ^ ((k % 4) * 2)).
          const int k = tt & 31;
          const int rbase = mn ? (tt >> 5) * 4096 + k * 128 : tt * 128;
          const int rxor = mn ? (k & 3) << 1 : (tt & 7);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            // bf16 chunk j of hi (and of lo): raw chunks 2j and 2j + 1
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int u = 0; u < 2; u++) {
              const float4 x = *reinterpret_cast<const float4 *>(sb + rbase + (((2 * j + u) ^ rxor) << 4));
              // hi = the tf32 part the hi*hi product uses, lo = the rest (exact
              // in fp32), each rounded to bf16
              const float h0 = tf32_trunc(x.x), h1 = tf32_trunc(x.y), h2 = tf32_trunc(x.z), h3 = tf32_trunc(x.w);
              hw[2 * u] = b2_bits(__floats2bfloat162_rn(h0, h1));
              hw[2 * u + 1] = b2_bits(__floats2bfloat162_rn(h2, h3));
              lw[2 * u] = b2_bits(__floats2bfloat162_rn(x.x - h0, x.y - h1));
              lw[2 * u + 1] = b2_bits(__floats2bfloat162_rn(x.z - h2, x.w - h3));
            }
            int hoff, loff;
            if (!mn) {
              // packed row r: hi chunks 0-3, lo chunks 4-7, chunk at c ^ (r % 8)
              hoff = tt * 128 + ((j ^ (tt & 7)) << 4);
              loff = tt * 128 + (((4 + j) ^ (tt & 7)) << 4);
            } else {
              // MN elements 32 * (tt / 32) + 8j.. of K row k: block (tt / 64),
              // chunk 4 * ((tt / 32) % 2) + j of the row, at chunk ^ (k % 8)
              const int blk = tt >> 6, ch = 4 * ((tt >> 5) & 1) + j;
              hoff = blk * 4096 + (k >> 3) * 1024 + (k & 7) * 128 + ((ch ^ (k & 7)) << 4);
              loff = hoff + 8192;
            }
            // A's concatenated K is [hi | lo], B's [lo | hi]
            const uint4 H4 = make_uint4(hw[0], hw[1], hw[2], hw[3]), L4 = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            *reinterpret_cast<uint4 *>(db + hoff) = is_a ? H4 : L4;
            *reinterpret_cast<uint4 *>(db + loff) = is_a ? L4 : H4;
          }
        } else {
          // A tile then this CTA's B half: 2048 float4 of raw data, 8 per
          // thread; lo lands at the same offset of the lo slot (same layout).
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const int off = (e * 256 + t) * 16;
            const float4 x = *reinterpret_cast<const float4 *>(src + off);
            float4 lo;
            lo.x = x.x - tf32_trunc(x.x); lo.y = x.y - tf32_trunc(x.y);
            lo.z = x.z - tf32_trunc(x.z); lo.w = x.w - tf32_trunc(x.w);
            *reinterpret_cast<float4 *>(dst + off) = lo;
          }
        }
        // Every writer orders its stores before the tensor pipe's reads.
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(cluster_map(bar_ready(ls), 0));
        kb++;
      }
    }
    if (ok && !*abort_flag) {
      const int row = i0 + q * 32 + lane;
      if (p.rope_cos && row < p.I) {
        // RoPE (tinylm.c:626-640): this thread's 128 columns are two heads;
        // pairs (i, i + 32) rotate by the angle of the row's position.
        const size_t tb = (size_t)(row % p.rope_T) * 32;
#pragma unroll
        for (int i4 = 0; i4 < 32; i4 += 4) {
          const float4 c4 = __ldg(reinterpret_cast<const float4 *>(p.rope_cos + tb + i4));
          const float4 s4 = __ldg(reinterpret_cast<const float4 *>(p.rope_sin + tb + i4));
          const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
          for (int u = 0; u < 4; u++) {
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
              const float a = acc[64 * hh + i4 + u], b = acc[64 * hh + i4 + u + 32];
              acc[64 * hh + i4 + u] = a * cc[u] - b * ss[u];
              acc[64 * hh + i4 + u + 32] = b * cc[u] + a * ss[u];
            }
          }
        }
      }
      const int jc = j0 + h * BN;
      if (row < p.I && tail_slot >= 0) {
        // a part of a tail tile: this row of the tile's slot, no addend
        float *dst = p.tail_ws + (size_t)tail_slot * (PM * PN) + (size_t)(row - pm * PM) * PN + h * BN;
        store_row(dst, nullptr, acc, p.J - jc);
      } else if (row < p.I) {
        float *dst = Cout + (size_t)row * p.ldc + jc;
        const float *addp = p.add ? p.add + (size_t)row * p.ldc + jc : nullptr;
        store_row(dst, addp, acc, p.J - jc);
      }
    }
  }
  // Neither CTA releases TMEM or exits while the pair's MMAs, TMEM reads or
  // cross-CTA signals may still be in flight.
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PAIR_TMEM_COLS) : "memory");
  }
}

// ------------------------------- CTA pair, fp16 split, specialised warps
// The fp16-split engine (kind::f16, twice the tf32 MMA rate) with its work
// spread over dedicated warps.  In the pair kernel above the same eight warps
// convert every landed tile and drain the TMEM accumulator, and at the f16
// MMA rate they become the bottleneck.  Here (512 threads, 4 warpgroups):
//   warp 0          TMA producer (raw fp32 tiles, as in the pair kernel)
//   warp 1          TMEM owner and, in the leader CTA, MMA issuer
//   warps 2-3, 12-15  six converter warps: scale, split and pack each landed
//                   raw tile into the fp16 hi/lo operand tile (the layouts of
//                   the pair kernel's fp16 path), in 16-byte tasks
//   warps 4-11      eight accumulator warps: drain every TMEM chunk into fp32
//                   registers (128 columns per thread) and store the tile
// Registers follow the roles (setmaxnreg): warpgroups 0 and 3 run with 56 per
// thread, warpgroups 1 and 2 (the accumulators) with 200; 128 x 56 x 2 +
// 256 x 200 = 512 x 128, the launch's own total.
constexpr int WS_THREADS = 512;
constexpr int WS_CONV_WARPS = 6;
constexpr int WS_DRAIN_WARPS = 8;
constexpr int WS_REG_SMALL = 56, WS_REG_ACC = 200;
static_assert(128 * WS_REG_SMALL * 2 + 256 * WS_REG_ACC == WS_THREADS * 128, "register split must match the launch");

// Accumulator warps (4..11) of the specialised fp16-split kernel: drain every
// TMEM chunk into fp32 registers, then scale, rotate (RoPE) and store the
// tile rows.
template <bool A_MN, bool B_MN>
__device__ __forceinline__ void ws_accumulate(const Params &p, uint32_t tmem, int warp, int lane, int i0, int j0,
                                              int pm, int nchunks, int tail_slot, float *Cout, uint64_t *bars,
                                              volatile int *abort_flag, uint32_t peer_flag, const float *scl) {
  auto bar_accf = [&](int b) { return smem_u32(&bars[2 * RAW_STAGES + 2 * LO_STAGES + b]); };
  auto bar_acce = [&](int b) { return smem_u32(&bars[2 * RAW_STAGES + 2 * LO_STAGES + 2 + b]); };
  const int q = warp & 3, h = (warp - 4) >> 2;
  float acc[BN];
#pragma unroll
  for (int e = 0; e < BN; e++) acc[e] = 0.0f;
  bool ok = true;
  for (int c = 0; c < nchunks; c++) {
    const int b = c & 1;
    const bool landed = mbar_wait_pair(bar_accf(b), (c >> 1) & 1, abort_flag, peer_flag, p.err, 5);
    if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
    tc_fence_after();
#pragma unroll
    for (int cc = 0; cc < BN / 32; cc++) {
      uint32_t v[32];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * PN + h * BN + cc * 32;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
            "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
            "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
            "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int e = 0; e < 32; e++) acc[cc * 32 + e] += __uint_as_float(v[e]);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(cluster_map(bar_acce(b), 0));
  }
  if (ok && !*abort_flag) {
    const float inv = scl[6];
#pragma unroll
    for (int e = 0; e < BN; e++) acc[e] *= inv;
    const int row = i0 + q * 32 + lane;
    if (p.rope_cos && row < p.I) {
      // RoPE (tinylm.c:626-640): this thread's 128 columns are two heads;
      // pairs (i, i + 32) rotate by the angle of the row's position.
      const size_t tb = (size_t)(row % p.rope_T) * 32;
#pragma unroll
      for (int i4 = 0; i4 < 32; i4 += 4) {
        const float4 c4 = __ldg(reinterpret_cast<const float4 *>(p.rope_cos + tb + i4));
        const float4 s4 = __ldg(reinterpret_cast<const float4 *>(p.rope_sin + tb + i4));
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int u = 0; u < 4; u++) {
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            const float a = acc[64 * hh + i4 + u], bb = acc[64 * hh + i4 + u + 32];
            acc[64 * hh + i4 + u] = a * cc[u] - bb * ss[u];
            acc[64 * hh + i4 + u + 32] = bb * cc[u] + a * ss[u];
          }
        }
      }
    }
    const int jc = j0 + h * BN;
    if (row < p.I && tail_slot >= 0) {
      float *dst = p.tail_ws + (size_t)tail_slot * (PM * PN) + (size_t)(row - pm * PM) * PN + h * BN;
      store_row(dst, nullptr, acc, p.J - jc);
    } else if (row < p.I) {
      float *dst = Cout + (size_t)row * p.ldc + jc;
      const float *addp = p.add ? p.add + (size_t)row * p.ldc + jc : nullptr;
      store_row(dst, addp, acc, p.J - jc);
    }
  }
}

template <bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(WS_THREADS, 1)
gemm_tc_pair_f16ws_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                          const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                          Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *raw_ring = smem, *lo_ring = smem + RAW_STAGES * RAW_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(lo_ring + LO_STAGES * RAW_BYTES);
  // bars: full[R], rempty[R] (this CTA's converters done with the raw slot),
  // ready[L] (both CTAs' operand slot written; leader's copy used), lempty[L]
  // (pair MMAs done with the operand slot), accf[2], acce[2] (leader's copy)
  constexpr int NBARS = 2 * RAW_STAGES + 2 * LO_STAGES + 4;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float *scl = reinterpret_cast<float *>(tmem_slot + 4);   // [A0, B0, A1, B1, A2, B2], inverse product scale

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  int L = blockIdx.x >> 1;
  int kb0 = blockIdx.z * p.kb_per_split, kb_len = p.kb_per_split;
  int tail_slot = -1;
  if (p.tail_splits > 1 && L >= p.full_tiles) {
    const int u = L - p.full_tiles;
    L = p.full_tiles + u / p.tail_splits;
    kb0 = (u % p.tail_splits) * p.tail_kb;
    kb_len = p.tail_kb;
    tail_slot = u;
  }
  int pm, tn;
  pair_tile(L, p.I, p.J, &pm, &tn);
  const int i0 = (2 * pm + (int)rank) * BM;
  const int j0 = tn * PN;
  const int jb = j0 + (int)rank * BN;
  const int nk_all = (p.R + BK - 1) / BK;
  const int nk = max(0, min(nk_all - kb0, kb_len));
  const int nchunks = (nk + PAIR_CHUNK_KB - 1) / PAIR_CHUNK_KB;
  float *const Cout = p.C + (size_t)blockIdx.z * p.split_stride;
  const uint32_t raw_base = smem_u32(raw_ring), lo_base = smem_u32(lo_ring);
  auto bar_full = [&](int s) { return smem_u32(&bars[s]); };
  auto bar_rempty = [&](int s) { return smem_u32(&bars[RAW_STAGES + s]); };
  auto bar_ready = [&](int s) { return smem_u32(&bars[2 * RAW_STAGES + s]); };
  auto bar_lempty = [&](int s) { return smem_u32(&bars[2 * RAW_STAGES + LO_STAGES + s]); };
  auto bar_accf = [&](int b) { return smem_u32(&bars[2 * RAW_STAGES + 2 * LO_STAGES + b]); };
  auto bar_acce = [&](int b) { return smem_u32(&bars[2 * RAW_STAGES + 2 * LO_STAGES + 2 + b]); };
  const uint32_t peer_flag = cluster_map(smem_u32((const void *)abort_flag), rank ^ 1u);

  if (threadIdx.x == 0) {
    for (int s = 0; s < RAW_STAGES; s++) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_rempty(s), WS_CONV_WARPS);
    }
    for (int s = 0; s < LO_STAGES; s++) {
      mbar_init(bar_ready(s), 2 * WS_CONV_WARPS);
      mbar_init(bar_lempty(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(bar_accf(b), 1);
      mbar_init(bar_acce(b), 2 * WS_DRAIN_WARPS);
    }
    *abort_flag = 0;
    // Operand scales as in the pair kernel's fp16 path.
    const int nprod = p.seg_end1 != 0x7fffffff ? 3 : (p.seg_end0 != 0x7fffffff ? 2 : 1);
    int P = 1 << 20;
#pragma unroll
    for (int t = 0; t < 3; t++)
      if (t < nprod) P = min(P, 28 - amax_exp(p.amax[2 * t]) - amax_exp(p.amax[2 * t + 1]));
    P = max(-126, min(126, P));
#pragma unroll
    for (int t = 0; t < 3; t++) {
      const int sb = t < nprod ? 14 - amax_exp(p.amax[2 * t + 1]) : 0;
      const int ea = t < nprod ? max(P - sb, -126) : 0;
      scl[2 * t] = exp2i(ea);
      scl[2 * t + 1] = t < nprod ? exp2i(P - ea) : 1.0f;
    }
    scl[6] = exp2i(-P);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(PAIR_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int wg = warp >> 2;
  // Each role's register budget is set at the top of its branch (the register
  // allocator sees the new limit for everything the branch dominates).
  if (wg == 1 || wg == 2) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(WS_REG_ACC));
    ws_accumulate<A_MN, B_MN>(p, tmem, warp, lane, i0, j0, pm, nchunks, tail_slot, Cout, bars, abort_flag,
                              peer_flag, scl);
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(WS_REG_SMALL));
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % RAW_STAGES, u = kb / RAW_STAGES;
        if (u > 0 && !mbar_wait_pair(bar_rempty(s), (u - 1) & 1, abort_flag, peer_flag, p.err, 1)) break;
        issued = kb + 1;
        const uint32_t st = raw_base + s * RAW_BYTES;
        mbar_arrive_expect_tx(bar_full(s), TX_BYTES);
        int kg = kb0 + kb;
        const CUtensorMap *ta = &tmA, *tb = &tmB;
        if (kg >= p.seg_end1) { ta = &tmA2; tb = &tmB2; kg -= p.seg_end1; }
        else if (kg >= p.seg_end0) { ta = &tmA1; tb = &tmB1; kg -= p.seg_end0; }
        const int k0 = kg * BK;
        if (A_MN) {
#pragma unroll
          for (int b = 0; b < BM / 32; b++) tma_load_2d(st + b * 4096, ta, bar_full(s), i0 + 32 * b, k0);
        } else {
          tma_load_2d(st, ta, bar_full(s), k0, i0);
        }
        if (B_MN) {
#pragma unroll
          for (int b = 0; b < BN / 32; b++) tma_load_2d(st + TILE_A + b * 4096, tb, bar_full(s), jb + 32 * b, k0);
        } else {
          tma_load_2d(st + TILE_A, tb, bar_full(s), k0, jb);
        }
      }
      for (int kb = issued > RAW_STAGES ? issued - RAW_STAGES : 0; kb < issued; kb++) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar_full(kb % RAW_STAGES), (kb / RAW_STAGES) & 1)) {
          if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicExch(p.err, 6); break; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (leader CTA only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc16 = make_idesc_pair_f16(A_MN, B_MN);
      int chunk = 0, kin = 0, last_committed = -1;
      for (int kb = 0; kb < nk; kb++) {
        const int ls = kb % LO_STAGES;
        const int b = chunk & 1;
        if (kin == 0 && chunk >= 2 &&
            !mbar_wait_pair(bar_acce(b), ((chunk >> 1) - 1) & 1, abort_flag, peer_flag, p.err, 7))
          break;
        if (!mbar_wait_pair(bar_ready(ls), (kb / LO_STAGES) & 1, abort_flag, peer_flag, p.err, 2)) break;
        tc_fence_after();
        const uint32_t lo = lo_base + ls * RAW_BYTES;
        const uint32_t d = tmem + b * PN;
#pragma unroll
        for (int kk = 0; kk < BK / 16; kk++) {
          uint64_t op[2][2];   // [A, B][hi, lo]
#pragma unroll
          for (int w = 0; w < 2; w++) {
            const bool mn = w ? B_MN : A_MN;
            const uint32_t t0 = lo + (w ? TILE_A : 0);
            op[w][0] = mn ? smem_desc(t0 + kk * 2048, 4096, 1024, LAYOUT_SW128)
                          : smem_desc(t0 + kk * 32, 16, 1024, LAYOUT_SW128);
            op[w][1] = mn ? smem_desc(t0 + 8192 + kk * 2048, 4096, 1024, LAYOUT_SW128)
                          : smem_desc(t0 + 64 + kk * 32, 16, 1024, LAYOUT_SW128);
          }
          tc_mma_pair_f16(d, op[0][1], op[1][0], idesc16, (kin > 0 || kk > 0) ? 1u : 0u);
          tc_mma_pair_f16(d, op[0][0], op[1][1], idesc16, 1);
          tc_mma_pair_f16(d, op[0][0], op[1][0], idesc16, 1);
        }
        tc_commit_pair(bar_lempty(ls));
        if (++kin == PAIR_CHUNK_KB || kb == nk - 1) {
          tc_commit_pair(bar_accf(b));
          last_committed = chunk;
          chunk++;
          kin = 0;
        }
      }
      if (kin > 0 || last_committed < chunk - 1 || last_committed < 0) {
        tc_commit_pair(bar_accf(chunk & 1));
        last_committed = chunk;
      }
      const int b = last_committed & 1;
      const long long t0 = clock64();
      while (!mbar_try_wait(bar_accf(b), (last_committed >> 1) & 1)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) { pair_abort(abort_flag, peer_flag, p.err, 3); break; }
      }
    }
  } else {
    // ------------------------- converter warps (2, 3, 12..15): 6 x 32 threads
    const int cw = warp < 4 ? warp - 2 : warp - 10;   // converter warp 0..5
    // Lane -> (row of an 8-row group, 16-byte chunk j): a quarter-warp (the
    // unit of a 16-byte shared-memory access) takes rows r and r ^ 5 of the
    // group, whose swizzled chunks fall in disjoint banks for the raw loads
    // and for the hi / lo stores of both layouts.
    const int qrow = (lane >> 3) ^ (((lane >> 2) & 1) ? 5 : 0), j = lane & 3;
    const int half = (lane >> 2) & 1;
    for (int kb = 0; kb < nk; kb++) {
      const int rs = kb % RAW_STAGES, ls = kb % LO_STAGES;
      bool landed = mbar_wait_pair(bar_full(rs), (kb / RAW_STAGES) & 1, abort_flag, peer_flag, p.err, 4);
      if (landed && kb >= LO_STAGES)
        landed = mbar_wait_pair(bar_lempty(ls), ((kb / LO_STAGES) - 1) & 1, abort_flag, peer_flag, p.err, 8);
      if (!__all_sync(0xffffffffu, landed)) break;
      const uint8_t *src = raw_ring + rs * RAW_BYTES;
      uint8_t *dst = lo_ring + ls * RAW_BYTES;
      const int kg = kb0 + kb;
      const int tp = kg >= p.seg_end1 ? 2 : (kg >= p.seg_end0 ? 1 : 0);
      const float sca = scl[2 * tp], scb = scl[2 * tp + 1];
      // Unit = 32 tasks = 8 raw rows x 4 chunks; task = (tile, raw row tt,
      // fp16 chunk j): 8 values of raw row tt (raw chunks 2j, 2j + 1) into hi
      // chunk j and lo chunk j.  Raw row: K-major row tt (chunk c at
      // c ^ (tt % 8)); MN-major box tt / 32, K row k = tt % 32 (chunk c at
      // c ^ ((k % 4) * 2)).  Units 0-15: A tile, 16-31: this CTA's B half.
      for (int unit = cw; unit < 32; unit += WS_CONV_WARPS) {
        const bool is_a = unit < 16, mn = is_a ? A_MN : B_MN;
        const int tt = (unit & 15) * 8 + qrow;
        const float sc = is_a ? sca : scb;
        const uint8_t *sb = src + (is_a ? 0 : TILE_A);
        uint8_t *db = dst + (is_a ? 0 : TILE_A);
        const int k = tt & 31;
        const int rbase = mn ? (tt >> 5) * 4096 + k * 128 : tt * 128;
        const int rxor = mn ? (k & 3) << 1 : (tt & 7);
        uint32_t hw[4], lw[4];
        // MN-major rows of a quarter-warp share the even (odd) chunks: the
        // second row of each quarter loads its odd chunk first.
        const int u0 = mn ? half : 0;
        const float4 xa = *reinterpret_cast<const float4 *>(sb + rbase + (((2 * j + u0) ^ rxor) << 4));
        const float4 xb = *reinterpret_cast<const float4 *>(sb + rbase + (((2 * j + (u0 ^ 1)) ^ rxor) << 4));
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const float4 x = (u == 0) == (u0 == 0) ? xa : xb;
          const float v0 = x.x * sc, v1 = x.y * sc, v2 = x.z * sc, v3 = x.w * sc;
          const float h0 = tf32_trunc(v0), h1 = tf32_trunc(v1), h2 = tf32_trunc(v2), h3 = tf32_trunc(v3);
          hw[2 * u] = h2_bits(__floats2half2_rn(h0, h1));
          hw[2 * u + 1] = h2_bits(__floats2half2_rn(h2, h3));
          lw[2 * u] = h2_bits(__floats2half2_rn(v0 - h0, v1 - h1));
          lw[2 * u + 1] = h2_bits(__floats2half2_rn(v2 - h2, v3 - h3));
        }
        int hoff, loff;
        if (!mn) {
          hoff = tt * 128 + ((j ^ (tt & 7)) << 4);
          loff = tt * 128 + (((4 + j) ^ (tt & 7)) << 4);
        } else {
          const int blk = tt >> 6, ch = 4 * ((tt >> 5) & 1) + j;
          hoff = blk * 4096 + (k >> 3) * 1024 + (k & 7) * 128 + ((ch ^ (k & 7)) << 4);
          loff = hoff + 8192;
        }
        *reinterpret_cast<uint4 *>(db + hoff) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(db + loff) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_remote(cluster_map(bar_ready(ls), 0));
        mbar_arrive(bar_rempty(rs));
      }
    }
  }
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PAIR_TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encoder() {
  if (g_encode) return TL_OK;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return set_error(TL_ECUDA, "cuTensorMapEncodeTiled not available from the driver");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return TL_OK;
}

// 2D fp32 map over a row-major [outer][inner] array with row stride `ld` floats.
// K-major tiles use the 16-byte-chunk 128B swizzle, MN-major tiles the
// 32-byte-chunk one (matching the descriptor layouts above).
static int make_map(CUtensorMap *m, const float *ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                    uint32_t box_outer, bool mn_major) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TL_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TL_OK;
}

// Largest |x| over up to six arrays (blockIdx.y picks one), as float bits in
// out[y], which is zero beforehand: non-negative floats order like unsigned
// integers, so atomicMax gives the same bits in any order.  NaN bits exceed
// infinity's and propagate as "not finite".
struct AmaxArgs {
  const float *p[6];
  size_t n[6];
};
__global__ void absmax_kernel(AmaxArgs a, unsigned *out) {
  const float *x = a.p[blockIdx.y];
  const size_t n = a.n[blockIdx.y];
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t n4 = (reinterpret_cast<uintptr_t>(x) & 15) ? 0 : n / 4;
  unsigned m = 0;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
    m = max(m, max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                   max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu)));
  }
  for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    m = max(m, __float_as_uint(__ldg(x + i)) & 0x7fffffffu);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ unsigned wm[32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? wm[threadIdx.x] : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0 && m) atomicMax(out + blockIdx.y, m);
  }
}

// C[i, j] = add[i, j] + sum_z ws[z][i][j], partials summed in z order (add may
// be nullptr or C itself).
__global__ void splitk_reduce_kernel(float *C, int ldc, const float *add, const float *__restrict__ ws,
                                     int splits, int I, int J) {
  const size_t total4 = (size_t)I * J / 4;
  const size_t stride = (size_t)I * J;
  for (size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x; q < total4; q += (size_t)gridDim.x * blockDim.x) {
    const size_t e = q * 4;
    const int i = (int)(e / J), j = (int)(e % J);
    float4 acc = reinterpret_cast<const float4 *>(ws)[q];
    for (int z = 1; z < splits; z++) {
      const float4 w = reinterpret_cast<const float4 *>(ws + z * stride)[q];
      acc.x += w.x; acc.y += w.y; acc.z += w.z; acc.w += w.w;
    }
    if (add) {
      const float4 o = *reinterpret_cast<const float4 *>(add + (size_t)i * ldc + j);
      acc.x = o.x + acc.x; acc.y = o.y + acc.y; acc.z = o.z + acc.z; acc.w = o.w + acc.w;
    }
    *reinterpret_cast<float4 *>(C + (size_t)i * ldc + j) = acc;
  }
}

// The tail tiles of a tail-split pair launch: C = add + the tile's parts
// summed in part order (add may be nullptr or C itself).  blockIdx.y = tail
// tile.
__global__ void tail_reduce_kernel(float *C, int ldc, const float *add, const float *__restrict__ ws, int full_tiles,
                                   int splits, int I, int J) {
  const int t = blockIdx.y;
  int pm, tn;
  pair_tile(full_tiles + t, I, J, &pm, &tn);
  const int r0 = pm * PM, c0 = tn * PN;
  const int rows = min(PM, I - r0), cols = min(PN, J - c0);
  const float *src0 = ws + (size_t)t * splits * (PM * PN);
  for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < PM * PN / 4; q += gridDim.x * blockDim.x) {
    const int r = q / (PN / 4), cc = (q % (PN / 4)) * 4;
    if (r >= rows || cc >= cols) continue;     // cols is a multiple of 4 (row strides of 16 bytes)
    const float *src = src0 + (size_t)r * PN + cc;
    float4 acc = *reinterpret_cast<const float4 *>(src);
    for (int z = 1; z < splits; z++) {
      const float4 w = *reinterpret_cast<const float4 *>(src + (size_t)z * (PM * PN));
      acc.x += w.x; acc.y += w.y; acc.z += w.z; acc.w += w.w;
    }
    const size_t o = (size_t)(r0 + r) * ldc + c0 + cc;
    if (add) {
      const float4 a4 = *reinterpret_cast<const float4 *>(add + o);
      acc.x = a4.x + acc.x; acc.y = a4.y + acc.y; acc.z = a4.z + acc.z; acc.w = a4.w + acc.w;
    }
    *reinterpret_cast<float4 *>(C + o) = acc;
  }
}

// CTA pairs of the pair kernel that can be resident at once on this device
// (clusters of two must sit on one GPC, so this can be below SMs / 2);
// 0 if unknown.
static int pair_slots(DeviceCtx *c) {
  static int slots[kMaxDevices] = {};
  if (slots[c->device]) return slots[c->device] > 0 ? slots[c->device] : 0;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2; attr.val.clusterDim.y = 1; attr.val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * 1024, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = PAIR_SMEM_BYTES;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_pair_kernel<false, true, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM_BYTES);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, gemm_tc_pair_kernel<false, true, false>, &cfg);
  if (e != cudaSuccess || n <= 0) {
    cudaGetLastError();
    slots[c->device] = -1;
    return 0;
  }
  slots[c->device] = n;
  return n;
}

template <bool A_MN, bool B_MN>
static int launch(DeviceCtx *c, const CUtensorMap &ma, const CUtensorMap &mb, const Params &p, int splits) {
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[c->device]) {
    TL_TRY_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     SMEM_BYTES));
    attr_set[c->device] = true;
  }
  dim3 grid((p.J + BN - 1) / BN, (p.I + BM - 1) / BM, splits);
  TraceScope ts(c, "gemm_tc");
  gemm_tc_kernel<A_MN, B_MN><<<grid, NUM_THREADS, SMEM_BYTES, c->stream>>>(ma, mb, p);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

// CTA pairs: grid x runs over the pairs' CTAs (cluster of 2 along x; the
// kernel maps pairs to output tiles in grouped order), z over K splits.
// SPLIT: the GemmSplit (tf32, fp16 on specialised warps, hybrid).
template <bool A_MN, bool B_MN, int SPLIT>
static int launch_pair(DeviceCtx *c, const CUtensorMap &ma, const CUtensorMap &mb, const Params &p, int splits,
                       const CUtensorMap *extra = nullptr) {
  constexpr bool F16 = SPLIT == (int)GemmSplit::F16, HYB = SPLIT == (int)GemmSplit::HYB;
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[c->device]) {
    if (F16)
      TL_TRY_CUDA(cudaFuncSetAttribute(gemm_tc_pair_f16ws_kernel<A_MN, B_MN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM_BYTES));
    else
      TL_TRY_CUDA(cudaFuncSetAttribute(gemm_tc_pair_kernel<A_MN, B_MN, HYB>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM_BYTES));
    attr_set[c->device] = true;
  }
  unsigned pairs = (unsigned)((p.I + PM - 1) / PM) * (unsigned)((p.J + PN - 1) / PN);
  if (p.tail_splits > 1) pairs = (unsigned)(p.full_tiles + (pairs - p.full_tiles) * p.tail_splits);
  dim3 grid(2 * pairs, 1, splits);
  TraceScope ts(c, "gemm_tc_pair");
  // extra: the maps of the second and third products (A1, B1, A2, B2)
  const CUtensorMap &a1 = extra ? extra[0] : ma, &b1 = extra ? extra[1] : mb;
  const CUtensorMap &a2 = extra ? extra[2] : ma, &b2 = extra ? extra[3] : mb;
  if (F16) {
    // The kernel moves registers between its warpgroups (setmaxnreg); the
    // split adds up to 128 per thread at launch.  A build with any other
    // launch count would wait forever in setmaxnreg.inc, so refuse it.
    static int regs[kMaxDevices] = {};
    if (!regs[c->device]) {
      cudaFuncAttributes fa;
      TL_TRY_CUDA(cudaFuncGetAttributes(&fa, gemm_tc_pair_f16ws_kernel<A_MN, B_MN>));
      regs[c->device] = fa.numRegs;
    }
    if (regs[c->device] != 128)
      return set_error(TL_EINVAL, "fp16-split kernel built with %d registers per thread, its register split needs 128",
                       regs[c->device]);
    gemm_tc_pair_f16ws_kernel<A_MN, B_MN><<<grid, WS_THREADS, PAIR_SMEM_BYTES, c->stream>>>(ma, mb, a1, b1, a2, b2, p);
  }
  else
    gemm_tc_pair_kernel<A_MN, B_MN, HYB><<<grid, NUM_THREADS, PAIR_SMEM_BYTES, c->stream>>>(ma, mb, a1, b1, a2, b2, p);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

}  // namespace tc

bool gemm_tc_supported(GemmOp op, const float *C, const float *A, const float *B, int M, int K, int N) {
  (void)op;
  const uintptr_t al = reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B);
  if (al & 15) return false;             // TMA needs 16-byte aligned bases
  if ((K & 3) || (N & 3)) return false;  // and row strides that are multiples of 16 bytes
  if (M < 1 || K < 1 || N < 1) return false;
  int I, J, R;
  gemm_dims(op, M, K, N, &I, &J, &R);
  if ((I + tc::BM - 1) / tc::BM > 65535) return false;
  if (2LL * ((I + tc::PM - 1) / tc::PM) * ((J + tc::PN - 1) / tc::PN) > 0x7fffffffLL) return false;
  return true;
}

// Everything the launches set up lazily on the host (driver entry point,
// shared-memory attributes), done ahead of a CUDA graph capture.
int gemm_tc_prepare(DeviceCtx *c) {
  int rc = tc::get_encoder();
  if (rc) return rc;
  (void)tc::pair_slots(c);
#define TL_PREP(K, BYTES) TL_TRY_CUDA(cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES))
  TL_PREP((tc::gemm_tc_kernel<false, true>), tc::SMEM_BYTES);
  TL_PREP((tc::gemm_tc_kernel<false, false>), tc::SMEM_BYTES);
  TL_PREP((tc::gemm_tc_kernel<true, true>), tc::SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_kernel<false, true, false>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_kernel<false, false, false>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_kernel<true, true, false>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_kernel<false, true, true>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_kernel<false, false, true>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_kernel<true, true, true>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_f16ws_kernel<false, true>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_f16ws_kernel<false, false>), tc::PAIR_SMEM_BYTES);
  TL_PREP((tc::gemm_tc_pair_f16ws_kernel<true, true>), tc::PAIR_SMEM_BYTES);
#undef TL_PREP
  return TL_OK;
}

bool gemm_tc_prefer_pair(int I, int J, int R) {
  (void)R;
  return I > tc::BM && J > tc::BN;
}

// Split-K choice, launch and (for s > 1) the fixed-order reduction of the
// partials, for an I x J output whose reduction runs over nk k-blocks read
// through the prepared tensor maps.  extra / seg_end0 / seg_end1: the maps
// and k-block boundaries of a second and third product summed into the same
// output (pair kernel, NT only).
// amax: the operand arrays of the fp16-split pair kernel (nullptr: another
// split); their max |x| is found first, on the stream, into the context's
// scratch.  hyb: the pair kernel with the hybrid split.
static int gemm_tc_launch(DeviceCtx *c, GemmOp op, float *C, int I, int J, int nk, int out_ldc,
                          const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap *extra, int seg_end0,
                          int seg_end1, bool pair, const float *add, const tc::AmaxArgs *amax, int namax,
                          bool hyb, const GemmRope *rope = nullptr) {
  tc::Params p;
  p.C = C; p.I = I; p.J = J; p.R = nk * tc::BK; p.err = c->err_flag;
  p.seg_end0 = seg_end0; p.seg_end1 = seg_end1;
  p.amax = nullptr;
  p.rope_cos = p.rope_sin = nullptr;
  p.rope_T = 1;
  if (rope) {
    p.rope_cos = rope->cosT; p.rope_sin = rope->sinT; p.rope_T = rope->T;
  }
  const bool f16 = pair && amax;
  if (f16) {
    size_t nmax = 0;
    for (int t = 0; t < namax; t++) nmax = std::max(nmax, amax->n[t]);
    TL_TRY_CUDA(cudaMemsetAsync(c->gemm_amax, 0, sizeof(unsigned) * 8, c->stream));
    TraceScope ts(c, "gemm_absmax");
    const unsigned bx = (unsigned)std::min<size_t>(std::max<size_t>((nmax / 4 + 255) / 256, 1), 2 * (size_t)c->num_sms);
    tc::absmax_kernel<<<dim3(bx, namax), 256, 0, c->stream>>>(*amax, c->gemm_amax);
    TL_TRY_CUDA(cudaGetLastError());
    p.amax = c->gemm_amax;
  }
  // Split-K.  A launch takes ceil(CTAs / SMs) waves of (k-blocks per split)
  // k-block times; splitting the reduction over s CTAs multiplies the CTAs by
  // s and divides the k-blocks by s, so the split count is chosen to minimise
  // waves * k-blocks plus the cost of the fixed-order reduction of the s
  // partials (s + 1 passes over the output at ~6 TB/s, ~1 us per k-block
  // time).  This fills the GPU for outputs with few tiles (weight gradients,
  // whose reduction runs over all tokens) and evens out the last wave.  Each
  // split gets whole TMEM chunks of k-blocks; partials go to the context's
  // workspace.  A pair tile (256 x 256) occupies two SMs.
  const int tm = pair ? tc::PM : tc::BM, tn = pair ? tc::PN : tc::BN, sms_per_tile = pair ? 2 : 1;
  const long long tiles = (long long)((I + tm - 1) / tm) * ((J + tn - 1) / tn);
  int splits = 1;
  double best = 0.0;           // cost of the chosen split, in k-block times
  if (c->gemm_ws && !rope) {   // (RoPE needs the whole sum in the epilogue)
    const size_t cap = c->gemm_ws_floats / ((size_t)I * J);
    const int smax = (int)std::min<size_t>(std::min(64, nk / tc::CHUNK_KB), cap);
    const double out_units = (double)I * J * 4.0 / 6.0e6;  // one output pass, in k-block times
    for (int s = 1; s <= std::max(1, smax); s++) {
      const long long ctas = tiles * sms_per_tile * s;
      const long long waves = (ctas + c->num_sms - 1) / c->num_sms;
      int kb = (nk + s - 1) / s;
      if (s > 1) kb = (kb + tc::CHUNK_KB - 1) / tc::CHUNK_KB * tc::CHUNK_KB;
      const double cost = (double)waves * kb + (s > 1 ? (s + 1) * out_units : 0.0);
      if (s == 1 || cost < best * 0.97) { best = cost; splits = s; }
    }
  }
  // Tail split (pair kernel): when the tiles fill `full` waves of co-resident
  // pairs and leave `rem` tiles for a last, partly empty wave, those rem
  // tiles run as ts pairs each over a ts-th of the reduction (ts = slots /
  // rem), their parts summed by a small fixed-order pass: the last wave then
  // takes 1/ts of a tile's time.  E.g. a 16384 x 1024 output: 256 tiles =
  // 3 waves of 74 pairs + 34 tiles; split 2 ways, 3.5 tile times instead of 4.
  p.full_tiles = 0; p.tail_splits = 1; p.tail_kb = 0; p.tail_ws = nullptr;
  if (pair && c->gemm_ws && !rope) {
    const int slots = tc::pair_slots(c);
    const long long full = slots > 0 ? tiles / slots * slots : tiles, rem = tiles - full;
    if (slots > 0 && rem > 0) {
      int ts = (int)std::min<long long>(slots / rem, nk / tc::PAIR_CHUNK_KB);
      ts = (int)std::min<size_t>(ts, c->gemm_ws_floats / ((size_t)rem * tc::PM * tc::PN));
      if (ts >= 2) {
        int tkb = (nk + ts - 1) / ts;
        tkb = (tkb + tc::PAIR_CHUNK_KB - 1) / tc::PAIR_CHUNK_KB * tc::PAIR_CHUNK_KB;
        ts = (nk + tkb - 1) / tkb;
        const double tail_units = (double)rem * (ts + 2) * tc::PM * tc::PN * 4.0 / 6.0e6;
        const double cost = (double)(full / slots) * nk + tkb + tail_units;
        if (ts >= 2 && cost < best * 0.97) {
          splits = 1;
          p.full_tiles = (int)full; p.tail_splits = ts; p.tail_kb = tkb; p.tail_ws = c->gemm_ws;
        }
      }
    }
  }
  int kb_per = nk;
  if (splits > 1) {
    kb_per = (nk + splits - 1) / splits;
    kb_per = (kb_per + tc::CHUNK_KB - 1) / tc::CHUNK_KB * tc::CHUNK_KB;
    splits = (nk + kb_per - 1) / kb_per;
  }
  p.kb_per_split = kb_per;
  if (splits > 1) {
    p.C = c->gemm_ws; p.ldc = J; p.add = nullptr; p.split_stride = (size_t)I * J;
  } else {
    p.ldc = out_ldc; p.add = add; p.split_stride = 0;
  }
  int rc = TL_OK;
  switch (op) {
    case GemmOp::NN:
      rc = !pair ? tc::launch<false, true>(c, ma, mb, p, splits)
           : f16 ? tc::launch_pair<false, true, (int)GemmSplit::F16>(c, ma, mb, p, splits)
           : hyb ? tc::launch_pair<false, true, (int)GemmSplit::HYB>(c, ma, mb, p, splits)
                 : tc::launch_pair<false, true, (int)GemmSplit::TF32>(c, ma, mb, p, splits);
      break;
    case GemmOp::NT:
      rc = !pair ? tc::launch<false, false>(c, ma, mb, p, splits)
           : f16 ? tc::launch_pair<false, false, (int)GemmSplit::F16>(c, ma, mb, p, splits, extra)
           : hyb ? tc::launch_pair<false, false, (int)GemmSplit::HYB>(c, ma, mb, p, splits, extra)
                 : tc::launch_pair<false, false, (int)GemmSplit::TF32>(c, ma, mb, p, splits, extra);
      break;
    case GemmOp::TN:
      rc = !pair ? tc::launch<true, true>(c, ma, mb, p, splits)
           : f16 ? tc::launch_pair<true, true, (int)GemmSplit::F16>(c, ma, mb, p, splits)
           : hyb ? tc::launch_pair<true, true, (int)GemmSplit::HYB>(c, ma, mb, p, splits)
                 : tc::launch_pair<true, true, (int)GemmSplit::TF32>(c, ma, mb, p, splits);
      break;
  }
  if (!rc && p.tail_splits > 1) {
    TraceScope ts(c, "gemm_tail_reduce");
    const int ntail = (int)(tiles - p.full_tiles);
    tc::tail_reduce_kernel<<<dim3(16, ntail), 256, 0, c->stream>>>(C, out_ldc, add, p.tail_ws, p.full_tiles,
                                                                  p.tail_splits, I, J);
    TL_TRY_CUDA(cudaGetLastError());
    return TL_OK;
  }
  if (rc || splits == 1) return rc;
  TraceScope ts(c, "gemm_splitk_reduce");
  const size_t q = (size_t)I * J / 4;
  unsigned blocks = (unsigned)std::min<size_t>((q + 255) / 256, (size_t)c->num_sms * 8);
  tc::splitk_reduce_kernel<<<blocks, 256, 0, c->stream>>>(C, out_ldc, add, c->gemm_ws, splits, I, J);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

int gemm_tc(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N, bool pair,
            const float *add, GemmSplit split, const GemmRope *rope) {
  const bool f16 = pair && split == GemmSplit::F16, hyb = pair && split == GemmSplit::HYB;
  int rc;
  if ((rc = tc::get_encoder())) return rc;
  int I, J, R;
  gemm_dims(op, M, K, N, &I, &J, &R);
  int out_ldc = 0;
  CUtensorMap ma, mb;
  switch (op) {
    case GemmOp::NN:  // A = X[M,K] K-major; B = W[K,N] MN-major
      out_ldc = N;
      if ((rc = tc::make_map(&ma, A, K, M, K, 32, tc::BM, false))) return rc;
      if ((rc = tc::make_map(&mb, B, N, K, N, 32, 32, true))) return rc;
      break;
    case GemmOp::NT:  // A = dY[M,N] K-major; B(r=n, j=k) = W[k*N+n] K-major
      out_ldc = K;
      if ((rc = tc::make_map(&ma, A, N, M, N, 32, tc::BM, false))) return rc;
      if ((rc = tc::make_map(&mb, B, N, K, N, 32, tc::BN, false))) return rc;
      break;
    case GemmOp::TN:  // A(i=k, r=m) = X[m*K+k] MN-major; B = dY[M,N] MN-major
      out_ldc = N;
      if ((rc = tc::make_map(&ma, A, K, M, K, 32, 32, true))) return rc;
      if ((rc = tc::make_map(&mb, B, N, M, N, 32, 32, true))) return rc;
      break;
  }
  const int nk = (R + tc::BK - 1) / tc::BK;
  tc::AmaxArgs am = {};
  am.p[0] = A; am.p[1] = B;
  switch (op) {   // the arrays' extents: A then B
    case GemmOp::NN: am.n[0] = (size_t)M * K; am.n[1] = (size_t)K * N; break;
    case GemmOp::NT: am.n[0] = (size_t)M * N; am.n[1] = (size_t)K * N; break;
    case GemmOp::TN: am.n[0] = (size_t)M * K; am.n[1] = (size_t)M * N; break;
  }
  return gemm_tc_launch(c, op, C, I, J, nk, out_ldc, ma, mb, nullptr, 0x7fffffff, 0x7fffffff, pair, add,
                        f16 ? &am : nullptr, 2, hyb, rope);
}

int gemm_tc_nt_sum(DeviceCtx *c, float *C, int nprod, const float *const *A, const float *const *B, const int *N,
                   int M, int K, GemmSplit split) {
  const bool f16 = split == GemmSplit::F16, hyb = split == GemmSplit::HYB;
  if (nprod < 1 || nprod > 3) return set_error(TL_EINVAL, "gemm_tc_nt_sum takes 1 to 3 products, not %d", nprod);
  int rc;
  if ((rc = tc::get_encoder())) return rc;
  // One pair of maps per product; product t covers k-blocks [end[t-1], end[t]).
  // A product's last k-block reads past its N columns, where the copies fill
  // zeros for both operands.
  CUtensorMap maps[6];
  int end[3];
  int nk = 0;
  for (int t = 0; t < nprod; t++) {
    if ((rc = tc::make_map(&maps[2 * t], A[t], N[t], M, N[t], 32, tc::BM, false))) return rc;
    if ((rc = tc::make_map(&maps[2 * t + 1], B[t], N[t], K, N[t], 32, tc::BN, false))) return rc;
    nk += (N[t] + tc::BK - 1) / tc::BK;
    end[t] = nk;
  }
  for (int t = nprod; t < 3; t++) {  // unused products: never reached
    maps[2 * t] = maps[0]; maps[2 * t + 1] = maps[1];
    end[t] = 0x7fffffff;
  }
  tc::AmaxArgs am = {};
  for (int t = 0; t < nprod; t++) {
    am.p[2 * t] = A[t]; am.n[2 * t] = (size_t)M * N[t];
    am.p[2 * t + 1] = B[t]; am.n[2 * t + 1] = (size_t)K * N[t];
  }
  return gemm_tc_launch(c, GemmOp::NT, C, M, K, nk, K, maps[0], maps[1], maps + 2, end[0], end[1], true, nullptr,
                        f16 ? &am : nullptr, 2 * nprod, hyb);
}

}  // namespace tl
