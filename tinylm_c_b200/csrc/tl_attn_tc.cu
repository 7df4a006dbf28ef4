// tl_attn_tc.cu -- causal GQA attention on the tensor cores (sm_100a), for
// T = 256 and head_dim 64: the forward (below), and the backward's key-side
// (dK, dV) and query-side (dQ) kernels further down, each with its own
// description.
//
// Forward, the reference's attn_fwd (tinylm.c:699-733): persistent CTA pairs
// (clusters of 2, tcgen05 cta_group::2), one per SM pair.  Pair p walks a
// contiguous range of (sequence, query head) items in (b, h) order, so the
// query heads of one kv-head group follow each other and share K, loaded and
// split once per group.  CTA r holds query rows 128r..128r+127 and key rows
// 128r..128r+127 of the item.
//
//   S = Q K^T      M = 256 queries, N = 256 keys, K = 64, on the hybrid split:
//                  hi*hi as 2 k-blocks x 4 tf32 MMAs on the raw tiles, the
//                  cross terms as 2 x 4 bf16 MMAs over K-concatenated rows
//                  (Q: [bf16(hi) | bf16(lo)], K: [bf16(lo) | bf16(hi)]), into
//                  TMEM buffer x = item % 2 (columns 256x..256x+255); Q and K
//                  staged by TMA (K-major, 128-byte swizzle), their bf16
//                  halves written by the softmax warps.
//   softmax        exact, two passes over S in TMEM: row max over the keys
//                  <= the query (the two column halves exchange partial maxima
//                  through shared memory), then p = 2^(s*scale*log2 e - max*log2 e)
//                  and the row sum.  P goes to shared memory in 32-key blocks
//                  (raw and lo, the A operand of the next product).
//   O = P V        M = 256, N = 64, K = 256 keys in 8 blocks through a 2-slot
//                  ring (P block + V block, V as the MN-major B operand: each
//                  CTA holds 32 of the 64 value columns), accumulated in TMEM
//                  over S's first 64 columns (key blocks 0 and 1, both read
//                  before the first product).
//   epilogue       out = O / rowsum, lse = max + log(rowsum) (what the backward
//                  kernels read).
// Overlap: Q of the next item is loaded as soon as this item's S products are
// done, split by the softmax warps after key block SPLIT_KB of this item's
// second pass, and the next S goes into the other TMEM buffer while this
// item's P V products and epilogue run; the next item's softmax starts from
// a finished S.
//
// Roles (320 threads): warp 0 lane 0 loads Q (and K), lane 1 the V blocks;
// warp 1 owns TMEM and, in the leader CTA, issues the MMAs; warps 2-9 split Q/K,
// run the softmax (warp w: TMEM lanes 32*(w%4).., h = (w-2)/4: row maximum
// over keys [128h, 128h+128), then P for the key blocks kb with kb % 2 == h
// and the lo parts of V for the others), then the epilogue for value columns
// [32h, 32h + 32).  Every wait is bounded; on expiry the pair records an error
// code (tl_device_status) and winds down.  No TMA multicast: the leader's
// commits use tcgen05.commit multicast, which moves no data.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdlib>
#include "tl_common.cuh"
#include "tl_tc_ptx.cuh"
#include "tl_trace.cuh"

namespace tl {
namespace atc {
using namespace tc;

constexpr int T = 256, HD = 64, QR = 128;       // sequence, head dim, query rows per CTA
constexpr int KBLK = 32;                        // floats per 128-byte swizzle row
constexpr int NKB = T / KBLK;                   // 8 key blocks
constexpr int TILE = QR * KBLK * 4;             // 16 KB: 128 rows x 32 floats
constexpr int OFF_QR = 0, OFF_QL = 2 * TILE, OFF_KR = 4 * TILE, OFF_KL = 6 * TILE;
constexpr int STAGE0 = 8 * TILE;                // Q, K (raw, lo; 2 k-blocks each): 128 KB
constexpr int VT = 32 * 32 * 4;                 // V box: 32 keys x 32 value columns, 4 KB
constexpr int OFF_PR = 0, OFF_PL = TILE, OFF_VR = 2 * TILE, OFF_VL = 2 * TILE + VT;
constexpr int STAGE_BYTES = 2 * TILE + 2 * VT;  // 40 KB
constexpr int NSTAGE = 2;
constexpr int NBARS = 16;
constexpr int SMEM_BYTES = STAGE0 + NSTAGE * STAGE_BYTES + 1024 /*align*/ + NBARS * 8 + 64 + 4 * QR * 4;
constexpr int NUM_THREADS = 320;
constexpr int TMEM_COLS = 512;                  // two S buffers of 256 columns (O over the first 64)
constexpr int SPLIT_KB = 3;                     // key block after which the next item's Q is split
constexpr int SIGNALLERS = 16;                  // split/softmax warps of the pair
static_assert(SMEM_BYTES <= 232448, "attention kernel exceeds the opt-in shared memory");

__host__ __device__ constexpr uint32_t idesc_m256(int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}
// the same shape with bf16 operands (kind::f16)
__host__ __device__ constexpr uint32_t idesc_m256_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// The bf16 K-concatenated operand of K-major tiles (rows of 32 floats, 128
// bytes, 16-byte chunks at c ^ (row % 8)): row r of dst holds bf16(hi) of its
// 32 values in chunks 0-3 and bf16(lo) in chunks 4-7, or lo first for a B
// operand; hi is the tf32 part the hi*hi product uses, lo = x - hi.  A task
// (row, j) turns raw chunks 2j, 2j + 1 into chunks j and 4 + j.
__device__ __forceinline__ uint32_t bf2_bits(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ void split_cat(const uint8_t *src, uint8_t *dst, int rows, bool lo_first, int t,
                                          int nthreads) {
  for (int task = t; task < rows * 4; task += nthreads) {
    const int r = task >> 2, j = task & 3, sw = r & 7;
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const float4 x = *reinterpret_cast<const float4 *>(src + r * 128 + (((2 * j + u) ^ sw) << 4));
      const float h0 = tf32_trunc(x.x), h1 = tf32_trunc(x.y), h2 = tf32_trunc(x.z), h3 = tf32_trunc(x.w);
      hw[2 * u] = bf2_bits(h0, h1);
      hw[2 * u + 1] = bf2_bits(h2, h3);
      lw[2 * u] = bf2_bits(x.x - h0, x.y - h1);
      lw[2 * u + 1] = bf2_bits(x.z - h2, x.w - h3);
    }
    const uint4 H4 = make_uint4(hw[0], hw[1], hw[2], hw[3]), L4 = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    *reinterpret_cast<uint4 *>(dst + r * 128 + ((j ^ sw) << 4)) = lo_first ? L4 : H4;
    *reinterpret_cast<uint4 *>(dst + r * 128 + (((4 + j) ^ sw) << 4)) = lo_first ? H4 : L4;
  }
}

// D (TMEM) (+)= A (shared memory) * B (shared memory), bf16 operands.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

struct Args {
  float *out, *lse;
  int H, KV, D;
  int items;                                    // B * H (sequence, query head) items
  float scale;
  int *err;
};

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGE0 + NSTAGE * STAGE_BYTES);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float *red = reinterpret_cast<float *>(tmem_slot + 16);   // [2 max/sum][2 halves][128 rows]
  const uint32_t base = smem_u32(smem);
  auto stage = [&](int s) { return base + STAGE0 + s * STAGE_BYTES; };
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // QK_FULL: Q (+ K) landed; QK_READY: their bf16 halves written (pair, leader's
  // copy); S_FULL[2]: S in TMEM buffer x complete (its Q/K also free again);
  // ST_FULL / ST_READY / ST_EMPTY [2]: V landed / P and V lo written / PV of
  // the stage done; O_FULL[2]: O in buffer x complete; O_EMPTY[2]: buffer x
  // read by the epilogue (pair, leader's copy); XCH: the two column halves'
  // row maxima and sums; FIN: every MMA done.
  constexpr int QK_FULL = 0, QK_READY = 1, S_FULL = 2, ST_FULL = 4, ST_READY = 6, ST_EMPTY = 8, O_FULL = 10,
                O_EMPTY = 12, XCH = 14, FIN = 15;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int grp = a.H / a.KV;
  // This pair's items: (sequence, query head) in (b, h) order, so consecutive
  // items of one kv-head group share K.
  const int npairs = (int)gridDim.x >> 1, pair = (int)blockIdx.x >> 1;
  const int it0 = (int)((long long)a.items * pair / npairs);
  const int n = (int)((long long)a.items * (pair + 1) / npairs) - it0;
  auto new_k = [&](int jl) { return jl == 0 || (it0 + jl) / grp != (it0 + jl - 1) / grp; };
  const uint32_t peer_flag = cluster_map(smem_u32((const void *)abort_flag), rank ^ 1u);

  if (threadIdx.x == 0) {
    mbar_init(bar(QK_FULL), 1);
    mbar_init(bar(QK_READY), SIGNALLERS);
    for (int x = 0; x < 2; x++) {
      mbar_init(bar(S_FULL + x), 1);
      mbar_init(bar(ST_FULL + x), 1);
      mbar_init(bar(ST_READY + x), SIGNALLERS);
      mbar_init(bar(ST_EMPTY + x), 1);
      mbar_init(bar(O_FULL + x), 1);
      mbar_init(bar(O_EMPTY + x), SIGNALLERS);
    }
    mbar_init(bar(XCH), 8);
    mbar_init(bar(FIN), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // -------------------------------------------- producer: Q (and K)
      int issued = 0;
      for (int jl = 0; jl < n; jl++) {
        const int it = it0 + jl, b = it / a.H, h = it % a.H, kvh = h / grp;
        // Q / K of the previous item are free once its S products are done.
        if (jl > 0 && !mbar_wait_pair(bar(S_FULL + ((jl - 1) & 1)), ((jl - 1) >> 1) & 1, abort_flag, peer_flag,
                                      a.err, 31))
          break;
        const bool nk = new_k(jl);
        const int row0 = b * T + QR * (int)rank;
        mbar_arrive_expect_tx(bar(QK_FULL), (nk ? 4 : 2) * TILE);
        for (int kb = 0; kb < 2; kb++) {
          tma_load_2d(base + OFF_QR + kb * TILE, &tmQ, bar(QK_FULL), h * HD + KBLK * kb, row0);
          if (nk) tma_load_2d(base + OFF_KR + kb * TILE, &tmK, bar(QK_FULL), kvh * HD + KBLK * kb, row0);
        }
        issued = jl + 1;
      }
      // No copy may still be landing when the CTA exits.
      if (issued > 0) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar(QK_FULL), (issued - 1) & 1)) {
          if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicExch(a.err, 36); break; }
        }
      }
    } else if (lane == 1) {
      // ------------------------------------------- producer: V blocks
      int issued = 0;
      bool ok = true;
      for (int jl = 0; jl < n && ok; jl++) {
        const int it = it0 + jl, b = it / a.H, kvh = (it % a.H) / grp;
        for (int kb = 0; kb < NKB; kb++) {
          const int g = jl * NKB + kb, s = g & 1, u = g >> 1;
          if (u > 0 && !mbar_wait_pair(bar(ST_EMPTY + s), (u - 1) & 1, abort_flag, peer_flag, a.err, 31)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(ST_FULL + s), VT);
          tma_load_2d(stage(s) + OFF_VR, &tmV, bar(ST_FULL + s), kvh * HD + 32 * (int)rank, b * T + KBLK * kb);
          issued = g + 1;
        }
      }
      for (int g = issued > NSTAGE ? issued - NSTAGE : 0; g < issued; g++) {
        const long long t1 = clock64();
        while (!mbar_try_wait(bar(ST_FULL + (g & 1)), (g >> 1) & 1)) {
          if (clock64() - t1 > WAIT_LIMIT_CYCLES) { atomicExch(a.err, 36); break; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (leader CTA only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_s = idesc_m256(256, false, false);
      constexpr uint32_t idesc_s_bf = idesc_m256_bf16(256);
      constexpr uint32_t idesc_o = idesc_m256(HD, false, true);
      // S = Q K^T of item jl into TMEM buffer jl % 2.
      auto issue_s = [&](int jl) -> bool {
        const int x = jl & 1;
        // Buffer x last held item jl - 2, whose O the epilogue must have read.
        if (jl >= 2 && !mbar_wait_pair(bar(O_EMPTY + x), ((jl - 2) >> 1) & 1, abort_flag, peer_flag, a.err, 30))
          return false;
        if (!mbar_wait_pair(bar(QK_READY), jl & 1, abort_flag, peer_flag, a.err, 32)) return false;
        tc_fence_after();
        const uint32_t d = tmem + 256 * x;
        // hi*hi: tf32 on the raw tiles; then hi*lo + lo*hi: one bf16 chain
        // over the concatenated rows ([hi | lo] of Q, [lo | hi] of K)
#pragma unroll
        for (int kb = 0; kb < 2; kb++) {
#pragma unroll
          for (int kk = 0; kk < KBLK / 8; kk++) {
            const uint32_t off = kb * TILE + kk * 32;
            tc_mma_pair(d, smem_desc(base + OFF_QR + off, 16, 1024, LAYOUT_SW128),
                        smem_desc(base + OFF_KR + off, 16, 1024, LAYOUT_SW128), idesc_s, (kb > 0 || kk > 0) ? 1u : 0u);
          }
        }
#pragma unroll
        for (int kb = 0; kb < 2; kb++) {
#pragma unroll
          for (int kc = 0; kc < 4; kc++) {
            const uint32_t off = kb * TILE + (kc >> 1) * 64 + (kc & 1) * 32;
            tc_mma_pair_f16(d, smem_desc(base + OFF_QL + off, 16, 1024, LAYOUT_SW128),
                            smem_desc(base + OFF_KL + off, 16, 1024, LAYOUT_SW128), idesc_s_bf, 1);
          }
        }
        tc_commit_pair(bar(S_FULL + x));
        return true;
      };
      bool ok = n > 0 && issue_s(0);
      for (int jl = 0; jl < n && ok; jl++) {
        const int x = jl & 1;
        // O overwrites S's first 64 columns (key blocks 0 and 1): both
        // blocks are read before the first P V product.
        for (int kb = 0; kb < NKB && ok; kb++) {
          const int g = jl * NKB + kb, s = g & 1;
          if (kb == 0)
            ok = mbar_wait_pair(bar(ST_READY + s), (g >> 1) & 1, abort_flag, peer_flag, a.err, 33) &&
                 mbar_wait_pair(bar(ST_READY + (s ^ 1)), ((g + 1) >> 1) & 1, abort_flag, peer_flag, a.err, 33);
          else if (kb != 1)
            ok = mbar_wait_pair(bar(ST_READY + s), (g >> 1) & 1, abort_flag, peer_flag, a.err, 33);
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = stage(s);
#pragma unroll
          for (int kk = 0; kk < KBLK / 8; kk++) {
            const uint64_t p_hi = smem_desc(st + OFF_PR + kk * 32, 16, 1024, LAYOUT_SW128);
            const uint64_t p_lo = smem_desc(st + OFF_PL + kk * 32, 16, 1024, LAYOUT_SW128);
            const uint64_t v_hi = smem_desc(st + OFF_VR + kk * 1024, 4096, 512, LAYOUT_SW128_BASE32B);
            const uint64_t v_lo = smem_desc(st + OFF_VL + kk * 1024, 4096, 512, LAYOUT_SW128_BASE32B);
            const uint32_t d = tmem + 256 * x;
            tc_mma_pair(d, p_lo, v_hi, idesc_o, (kb > 0 || kk > 0) ? 1u : 0u);
            tc_mma_pair(d, p_hi, v_lo, idesc_o, 1);
            tc_mma_pair(d, p_hi, v_hi, idesc_o, 1);
          }
          tc_commit_pair(bar(ST_EMPTY + s));
          // The next item's S, while this item's softmax runs on.
          if (kb == SPLIT_KB && jl + 1 < n) ok = issue_s(jl + 1);
        }
        if (ok) tc_commit_pair(bar(O_FULL + x));
      }
      // Every issued MMA finished (also on the abort path) before TMEM is
      // released.
      tc_commit_pair(bar(FIN));
      const long long t0 = clock64();
      while (!mbar_try_wait(bar(FIN), 0)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) { pair_abort(abort_flag, peer_flag, a.err, 34); break; }
      }
    }
  } else {
    // --------------------------- split, softmax and epilogue (warps 2..9)
    const int t = threadIdx.x - 64;             // 0..255
    const int q4 = warp & 3, hh = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;                // this thread's query row in the CTA
    const int qpos = QR * (int)rank + r;         // its position in the sequence
    const int tl = q4 * 32 + lane;               // 0..127 within the half
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    const float c2 = a.scale * 1.4426950408889634f;   // scale * log2(e)
    // This thread's share of the bf16 halves of the landed Q (and K) tiles:
    // Q (the A operand) as [hi | lo] rows, K (B) as [lo | hi].
    auto split_qk = [&](int jl) -> bool {
      const bool landed = mbar_wait_pair(bar(QK_FULL), jl & 1, abort_flag, peer_flag, a.err, 35);
      if (!__all_sync(0xffffffffu, landed)) return false;
      split_cat(smem + OFF_QR, smem + OFF_QL, 2 * QR, false, t, 256);
      if (new_k(jl)) split_cat(smem + OFF_KR, smem + OFF_KL, 2 * QR, true, t, 256);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(cluster_map(bar(QK_READY), 0));
      return true;
    };
    bool ok = n > 0 && split_qk(0);
    for (int jl = 0; jl < n && ok; jl++) {
      const int it = it0 + jl, b = it / a.H, h = it % a.H, x = jl & 1;
      const uint32_t sbase = tmem + lane_addr + 256 * x;
      float m = -1e30f, lsum = 0.0f;
      ok = __all_sync(0xffffffffu, mbar_wait_pair(bar(S_FULL + x), (jl >> 1) & 1, abort_flag, peer_flag, a.err, 37));
      if (!ok) break;
      {
        // pass 1: partial row max over this half's keys <= qpos (keys of
        // the upper half are all masked for the first 128 queries)
        tc_fence_after();
        float mx = -1e30f;
        if (!(rank == 0 && hh == 1)) {
#pragma unroll 1
          for (int c = 0; c < 4; c++) {
            uint32_t v[32];
            const int j0 = hh * 128 + c * 32;
            tmem_ld32(sbase + j0, v);
#pragma unroll
            for (int e = 0; e < 32; e++)
              if (j0 + e <= qpos) mx = fmaxf(mx, __uint_as_float(v[e]));
          }
        }
        red[hh * QR + r] = mx;
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(XCH));
        ok = __all_sync(0xffffffffu, mbar_wait_pair(bar(XCH), 0, abort_flag, peer_flag, a.err, 38));
        if (!ok) break;
        m = fmaxf(red[r], red[QR + r]) * a.scale;
      }
      const float mc = m * 1.4426950408889634f;
      // pass 2: key blocks in order; half h writes P for the blocks kb with
      // kb % 2 == h and the lo parts of V for the others, so both halves
      // produce P blocks at the same time.  After block SPLIT_KB every warp
      // also splits its share of the next item's Q (and K).
#pragma unroll 1
      for (int kb = 0; kb < NKB && ok; kb++) {
        const int g = jl * NKB + kb, s = g & 1;
        const uint32_t st = stage(s);
        if ((kb & 1) == hh) {
          bool w = true;
          if (g >= 2) w = mbar_wait_pair(bar(ST_EMPTY + s), ((g >> 1) - 1) & 1, abort_flag, peer_flag, a.err, 39);
          if (!(ok = __all_sync(0xffffffffu, w))) break;
          tc_fence_after();
          float pr[32];
          if (kb * 32 > QR * (int)rank + QR - 1) {
            // every key of the block is after every query of this CTA
#pragma unroll
            for (int e = 0; e < 32; e++) pr[e] = 0.0f;
          } else {
            uint32_t v[32];
            tmem_ld32(sbase + kb * 32, v);
#pragma unroll
            for (int e = 0; e < 32; e++) {
              const int key = kb * 32 + e;
              pr[e] = key <= qpos ? exp2f(fmaf(__uint_as_float(v[e]), c2, -mc)) : 0.0f;
              lsum += pr[e];
            }
          }
          // row r of the 128 x 32 K-major tile: logical chunk c at c ^ (r % 8)
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const uint32_t off = (uint32_t)r * 128 + (uint32_t)((c ^ (r & 7)) * 16);
            const float4 xv = make_float4(pr[4 * c], pr[4 * c + 1], pr[4 * c + 2], pr[4 * c + 3]);
            float4 lo;
            lo.x = xv.x - tf32_trunc(xv.x); lo.y = xv.y - tf32_trunc(xv.y);
            lo.z = xv.z - tf32_trunc(xv.z); lo.w = xv.w - tf32_trunc(xv.w);
            *reinterpret_cast<float4 *>(smem + (st - base) + OFF_PR + off) = xv;
            *reinterpret_cast<float4 *>(smem + (st - base) + OFF_PL + off) = lo;
          }
        } else {
          const bool w = mbar_wait_pair(bar(ST_FULL + s), (g >> 1) & 1, abort_flag, peer_flag, a.err, 40);
          if (!(ok = __all_sync(0xffffffffu, w))) break;
#pragma unroll
          for (int e = 0; e < 2; e++) {
            const int off = (e * 128 + tl) * 16;
            const float4 xv = *reinterpret_cast<const float4 *>(smem + (st - base) + OFF_VR + off);
            float4 lo;
            lo.x = xv.x - tf32_trunc(xv.x); lo.y = xv.y - tf32_trunc(xv.y);
            lo.z = xv.z - tf32_trunc(xv.z); lo.w = xv.w - tf32_trunc(xv.w);
            *reinterpret_cast<float4 *>(smem + (st - base) + OFF_VL + off) = lo;
          }
        }
        tc_fence_before();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(cluster_map(bar(ST_READY + s), 0));
        if (kb == SPLIT_KB && jl + 1 < n) ok = split_qk(jl + 1);
      }
      if (!ok) break;
      // row sum: both halves, added in half order
      red[2 * QR + hh * QR + r] = lsum;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(XCH));
      ok = __all_sync(0xffffffffu, mbar_wait_pair(bar(XCH), 1, abort_flag, peer_flag, a.err, 41));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait_pair(bar(O_FULL + x), (jl >> 1) & 1, abort_flag, peer_flag,
                                                          a.err, 42));
      if (!ok || *abort_flag) break;
      const float l = red[2 * QR + r] + red[3 * QR + r];
      const float inv = 1.0f / l;
      tc_fence_after();
      uint32_t v[32];
      tmem_ld32(sbase + hh * 32, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(cluster_map(bar(O_EMPTY + x), 0));
      const int b_row = b * T + qpos;
      float *dst = a.out + (size_t)b_row * a.D + h * HD + hh * 32;
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        *reinterpret_cast<float4 *>(dst + e) =
            make_float4(__uint_as_float(v[e]) * inv, __uint_as_float(v[e + 1]) * inv,
                        __uint_as_float(v[e + 2]) * inv, __uint_as_float(v[e + 3]) * inv);
      if (hh == 0) a.lse[(size_t)it * T + qpos] = m + logf(l);
    }
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// RoPE's backward on one head row held in registers (64 values): the pair
// (i, i + 32) rotated by the transposed matrix, in the order the separate
// RoPE kernel uses.
__device__ __forceinline__ void rope_back_row(float (&v)[HD], const float *cs, const float *sn) {
#pragma unroll
  for (int i4 = 0; i4 < HD / 2; i4 += 4) {
    const float4 c = __ldg(reinterpret_cast<const float4 *>(cs + i4));
    const float4 s = __ldg(reinterpret_cast<const float4 *>(sn + i4));
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float a = v[i4 + u], b = v[i4 + u + HD / 2];
      v[i4 + u] = a * cc[u] + b * ss[u];
      v[i4 + u + HD / 2] = -a * ss[u] + b * cc[u];
    }
  }
}

// ------------------------------------------------------------- dQ = dS K
// The query-side product of the backward (tinylm.c:772-777, dq += dsc * k).
// An item is one (sequence, query head, query half r): M = 128 queries,
// N = 64, the reduction over keys [0, 128(r+1)) in blocks of 32.  A = dS
// comes from the key-side kernel's dS^T scratch ([b][h][key][query], queries
// contiguous, so the MN-major A operand), B = K (MN-major B), both by TMA
// with the 32-byte atom swizzle.  The scratch's tiles above the diagonal are
// never written by the key-side kernel and stay zero from the model's set-up,
// which covers the 64-key tile above the diagonal inside each 128 x 128 block
// read here.
// Persistent: one CTA per SM walks items it, it + grid, ... (the halves with
// 8 key blocks first, then those with 4), through a ring of four stages that
// runs on across items, so the next item's loads and products overlap this
// item's epilogue.  Key blocks 0-3 accumulate in TMEM columns 0..63 of the
// item's buffer and 4-7 in 64..127 (each sum kept short in the truncating
// TMEM adds), added in fp32 by the epilogue; items alternate between two
// buffers of 128 columns.
// Roles (320 threads): warp 0 TMA producer, warp 1 TMEM owner and MMA issuer,
// warps 2-5 lo split of every stage, warps 6-9 the epilogue (warp w: rows
// 32*(w%4)..).  Every wait is bounded; on expiry the CTA records an error
// code (tl_device_status) and winds down.
constexpr int DQ_KB = 32;
constexpr int DQ_TILE_A = QR * DQ_KB * 4;                       // 16 KB: 4 boxes of 32 queries x 32 keys
constexpr int DQ_TILE_B = HD * DQ_KB * 4;                       // 8 KB: 2 boxes of 32 columns x 32 keys
constexpr int DQ_OFF_AHI = 0, DQ_OFF_ALO = DQ_TILE_A, DQ_OFF_BHI = 2 * DQ_TILE_A,
              DQ_OFF_BLO = 2 * DQ_TILE_A + DQ_TILE_B;
constexpr int DQ_STAGE_BYTES = 2 * (DQ_TILE_A + DQ_TILE_B);     // 48 KB
constexpr int DQ_STAGES = 4;
constexpr int DQ_THREADS = 320;
constexpr int DQ_NBARS = 3 * DQ_STAGES + 5;
constexpr int DQ_SMEM_BYTES = DQ_STAGES * DQ_STAGE_BYTES + 1024 + DQ_NBARS * 8 + 16;
constexpr int DQ_TMEM_COLS = 256;                               // two item accumulators of 128 columns
constexpr uint32_t DQ_IDESC = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 15) | (1u << 16) |
                              ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(QR >> 4) << 24);
static_assert(DQ_SMEM_BYTES <= 232448, "dQ kernel exceeds the opt-in shared memory");

struct DqArgs {
  float *dq;
  const float *cosT, *sinT;   // RoPE table [T][HD/2]: the inverse rotation is applied to dQ; nullptr: none
  int B, H, KV, D;
  int *err;
};

// Item it of 2 * B * H: the halves with 8 key blocks (r = 1) first.
struct DqItem {
  int r, bh, b, h, kvh, nk;
};
__device__ __forceinline__ DqItem dq_item(const DqArgs &a, int it) {
  DqItem d;
  const int BH = a.B * a.H;
  d.r = it < BH ? 1 : 0;
  d.bh = it < BH ? it : it - BH;
  d.b = d.bh / a.H;
  d.h = d.bh % a.H;
  d.kvh = d.h / (a.H / a.KV);
  d.nk = 4 * (d.r + 1);
  return d;
}

__global__ void __launch_bounds__(DQ_THREADS, 1)
attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmK, DqArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + DQ_STAGES * DQ_STAGE_BYTES);
  // bars: full[S] (TMA landed), ready[S] (lo parts written), empty[S] (MMAs
  // done with the stage), accf[2] (item's products in buffer b done),
  // acce[2] (epilogue done reading buffer b), fin (every MMA done)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + DQ_NBARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const uint32_t base = smem_u32(smem);
  auto bar_full = [&](int s) { return smem_u32(&bars[s]); };
  auto bar_ready = [&](int s) { return smem_u32(&bars[DQ_STAGES + s]); };
  auto bar_empty = [&](int s) { return smem_u32(&bars[2 * DQ_STAGES + s]); };
  auto bar_accf = [&](int b) { return smem_u32(&bars[3 * DQ_STAGES + b]); };
  auto bar_acce = [&](int b) { return smem_u32(&bars[3 * DQ_STAGES + 2 + b]); };
  const uint32_t bar_fin = smem_u32(&bars[3 * DQ_STAGES + 4]);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nitems = 2 * a.B * a.H;

  if (threadIdx.x == 0) {
    for (int s = 0; s < DQ_STAGES; s++) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_ready(s), 4);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(bar_accf(b), 1);
      mbar_init(bar_acce(b), 4);
    }
    mbar_init(bar_fin, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(DQ_TMEM_COLS)
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
      int g = 0;
      bool live = true;
      for (int it = blockIdx.x; live && it < nitems; it += gridDim.x) {
        const DqItem d = dq_item(a, it);
        for (int kb = 0; kb < d.nk; kb++, g++) {
          const int s = g % DQ_STAGES, u = g / DQ_STAGES;
          if (u > 0 && !mbar_wait(bar_empty(s), (u - 1) & 1, abort_flag, a.err, 51)) { live = false; break; }
          const uint32_t st = base + s * DQ_STAGE_BYTES;
          mbar_arrive_expect_tx(bar_full(s), DQ_TILE_A + DQ_TILE_B);
          const int key0 = kb * DQ_KB;
#pragma unroll
          for (int x = 0; x < QR / 32; x++)
            tma_load_2d(st + DQ_OFF_AHI + x * 4096, &tmS, bar_full(s), QR * d.r + 32 * x, d.bh * T + key0);
#pragma unroll
          for (int x = 0; x < HD / 32; x++)
            tma_load_2d(st + DQ_OFF_BHI + x * 4096, &tmK, bar_full(s), d.kvh * HD + 32 * x, d.b * T + key0);
        }
      }
      // No copy may still be landing when the CTA exits: the last
      // min(g, stages) issued stages.
      for (int q = g > DQ_STAGES ? g - DQ_STAGES : 0; q < g; q++) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar_full(q % DQ_STAGES), (q / DQ_STAGES) & 1)) {
          if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicExch(a.err, 56); break; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int g = 0, j = 0;
      bool live = true;
      for (int it = blockIdx.x; live && it < nitems; it += gridDim.x, j++) {
        const DqItem d = dq_item(a, it);
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(bar_acce(b), ((j >> 1) - 1) & 1, abort_flag, a.err, 57)) break;
        for (int kb = 0; kb < d.nk; kb++, g++) {
          const int s = g % DQ_STAGES, u = g / DQ_STAGES;
          if (!mbar_wait(bar_ready(s), u & 1, abort_flag, a.err, 52)) { live = false; break; }
          tc_fence_after();
          const uint32_t st = base + s * DQ_STAGE_BYTES;
          const uint32_t dt = tmem + (uint32_t)(b * 2 * HD + (kb >> 2) * HD);
#pragma unroll
          for (int kk = 0; kk < DQ_KB / 8; kk++) {
            const uint32_t off = kk * 1024;        // eight key rows per MMA step
            const uint64_t a_hi = smem_desc(st + DQ_OFF_AHI + off, 4096, 512, LAYOUT_SW128_BASE32B);
            const uint64_t a_lo = smem_desc(st + DQ_OFF_ALO + off, 4096, 512, LAYOUT_SW128_BASE32B);
            const uint64_t b_hi = smem_desc(st + DQ_OFF_BHI + off, 4096, 512, LAYOUT_SW128_BASE32B);
            const uint64_t b_lo = smem_desc(st + DQ_OFF_BLO + off, 4096, 512, LAYOUT_SW128_BASE32B);
            tc_mma(dt, a_lo, b_hi, DQ_IDESC, ((kb & 3) > 0 || kk > 0) ? 1u : 0u);
            tc_mma(dt, a_hi, b_lo, DQ_IDESC, 1);
            tc_mma(dt, a_hi, b_hi, DQ_IDESC, 1);
          }
          tc_commit(bar_empty(s));
        }
        if (!live) break;
        tc_commit(bar_accf(b));
      }
      // Every issued MMA finished (also on the abort path) before TMEM is
      // released and the CTA exits.
      tc_commit(bar_fin);
      const long long t0 = clock64();
      while (!mbar_try_wait(bar_fin, 0)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) { *abort_flag = 1; atomicExch(a.err, 55); break; }
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------- lo split (warps 2-5)
    const int t = threadIdx.x - 64;            // 0..127
    int g = 0;
    bool live = true;
    for (int it = blockIdx.x; live && it < nitems; it += gridDim.x) {
      const int nk = 4 * ((it < a.B * a.H ? 1 : 0) + 1);
      for (int kb = 0; kb < nk; kb++, g++) {
        const int s = g % DQ_STAGES, u = g / DQ_STAGES;
        const bool landed = mbar_wait(bar_full(s), u & 1, abort_flag, a.err, 53);
        if (!__all_sync(0xffffffffu, landed)) { live = false; break; }
        uint8_t *st = smem + s * DQ_STAGE_BYTES;
        // A then B: 1024 + 512 float4 of raw data, 12 per thread; lo lands at
        // the same offset of the lo tile (same swizzled layout).
#pragma unroll 4
        for (int e = 0; e < 12; e++) {
          const int idx = e * 128 + t;
          const int off = idx < 1024 ? DQ_OFF_AHI + idx * 16 : DQ_OFF_BHI + (idx - 1024) * 16;
          const int lo_off = off + (idx < 1024 ? DQ_TILE_A : DQ_TILE_B);
          const float4 x = *reinterpret_cast<const float4 *>(st + off);
          float4 lo;
          lo.x = x.x - tf32_trunc(x.x); lo.y = x.y - tf32_trunc(x.y);
          lo.z = x.z - tf32_trunc(x.z); lo.w = x.w - tf32_trunc(x.w);
          *reinterpret_cast<float4 *>(st + lo_off) = lo;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_ready(s));
      }
    }
  } else {
    // ------------------------------------------------- epilogue (warps 6-9)
    const int q4 = warp & 3, row = q4 * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    int j = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x, j++) {
      const DqItem d = dq_item(a, it);
      const int b = j & 1;
      const bool landed = mbar_wait(bar_accf(b), (j >> 1) & 1, abort_flag, a.err, 54);
      if (!__all_sync(0xffffffffu, landed) || *abort_flag) break;
      const int qpos = QR * d.r + row;
      if (a.cosT) {
        // this row's RoPE table entries into L1 while TMEM is read
        asm volatile("prefetch.global.L1 [%0];" ::"l"(a.cosT + (size_t)qpos * (HD / 2)));
        asm volatile("prefetch.global.L1 [%0];" ::"l"(a.sinT + (size_t)qpos * (HD / 2)));
      }
      tc_fence_after();
      float o[HD];
      const uint32_t tb = tmem + lane_addr + (uint32_t)(b * 2 * HD);
#pragma unroll
      for (int cc = 0; cc < HD / 32; cc++) {
        uint32_t v0[32];
        tmem_ld32(tb + cc * 32, v0);
#pragma unroll
        for (int e = 0; e < 32; e++) o[32 * cc + e] = __uint_as_float(v0[e]);
        if (d.r == 1) {
          uint32_t v1[32];
          tmem_ld32(tb + HD + cc * 32, v1);
#pragma unroll
          for (int e = 0; e < 32; e++) o[32 * cc + e] += __uint_as_float(v1[e]);
        }
      }
      // The buffer is free for the item after next as soon as it is read.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acce(b));
      // The gradient through RoPE (tinylm.c:1132-1133): the transposed
      // rotation of each (i, i + HD/2) pair at this query's position.
      if (a.cosT) rope_back_row(o, a.cosT + (size_t)qpos * (HD / 2), a.sinT + (size_t)qpos * (HD / 2));
      float *dst = a.dq + ((size_t)d.b * T + qpos) * a.D + (size_t)d.h * HD;
#pragma unroll
      for (int e = 0; e < HD; e += 4)
        *reinterpret_cast<float4 *>(dst + e) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(DQ_TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------- dK, dV (key side)
// The key-side products of the backward (tinylm.c:761-777: dv += p dO and
// dk += dsc q, with the scores and probabilities recomputed as at 748-758)
// for one (sequence, kv head, key block kb of 128 keys), looping over the
// group's query heads and the 32-query chunks at or after the key block.
// M = 128 keys throughout (cta_group::1):
//   S^T = K Q_c^T, dP^T = V dO_c^T   N = 32 queries, K = 64 in two blocks,
//        hybrid split: one tf32 product of the raw tiles (hi*hi) and the two
//        cross terms as one bf16 chain over K-concatenated tiles, A as
//        [bf16(hi) | bf16(lo)] and B as [bf16(lo) | bf16(hi)] per 128-byte
//        row (16 MMAs per product instead of 24, and a third fewer re-reads
//        of the A tile through shared memory); K and V stay resident
//        (K-major, raw and concatenated), Q_c and dO_c arrive by TMA as
//        K-major B tiles; into TMEM buffer i % 2 of chunk i.
//   P^T = exp(scale s - lse), dS^T = P^T (dP^T - D) scale   (warps 2-5, a key
//        row per thread): raw and lo parts written back to TMEM (P over S,
//        dS over dP), and dS^T to the scratch the dQ product reads.
//   dV += P^T dO_c, dK += dS^T Q_c   A from TMEM, B = dO_c / Q_c as MN-major
//        tiles (a second TMA copy, 32-byte atom swizzle), N = 64, K = 32; into
//        the accumulator pair of the current head (two, alternating by head),
//        which warps 6-9 add into fp32 registers once the head is done.
// The chunk tiles land in two raw buffers per kind (chunk i in buffer i % 2,
// so the next chunk's copies are in flight while this one is used) and have
// one converted buffer per kind (bf16 halves for the K-major tiles, tf32 lo
// parts for the MN-major ones), written once the previous chunk's products
// are done with it.  Roles (384 threads): warp 0 lane 0 loads K, V and the
// K-major tiles, lane 1 the MN-major tiles; warp 1 owns TMEM and issues the
// MMAs; warps 2-5 P and dS; warps 6-9 the bf16 halves of K and V, the lo
// parts of the MN-major tiles, and the per-head dV / dK sums; warps 10-11
// the bf16 halves of the K-major tiles.  Every wait is bounded.
constexpr int BW_THREADS = 384;
constexpr int BW_NQ = 32;                               // queries per chunk
constexpr int BW_KTILE = QR * 32 * 4;                   // 16 KB: 128 keys x 32 of head_dim
constexpr int BW_CTILE = BW_NQ * 32 * 4;                // 4 KB: 32 queries x 32 of head_dim
constexpr int BW_OFF_K = 0, BW_OFF_V = 4 * BW_KTILE;    // raw (2 tiles), then bf16 [hi | lo] (2 tiles): +32 KB
constexpr int BW_KV_LO = 2 * BW_KTILE;
// A chunk buffer: Q (2 tiles of 32 head_dim columns), then dO (2 tiles).
constexpr int BW_CBUF = 4 * BW_CTILE;                   // 16 KB
constexpr int BW_CB_O = 2 * BW_CTILE;                   // dO's offset in a chunk buffer
constexpr int BW_OFF_KMR = 8 * BW_KTILE;                // K-major raw buffers 0, 1
constexpr int BW_OFF_KML = BW_OFF_KMR + 2 * BW_CBUF;    // K-major bf16 [lo | hi]
constexpr int BW_OFF_MNR = BW_OFF_KML + BW_CBUF;        // MN-major raw buffers 0, 1
constexpr int BW_OFF_MNL = BW_OFF_MNR + 2 * BW_CBUF;    // MN-major lo
constexpr int BW_DATA = BW_OFF_MNL + BW_CBUF;           // 224 KB
constexpr int BW_NBARS = 21;
constexpr int BW_SMEM_BYTES = BW_DATA + 1024 + BW_NBARS * 8 + 16;
static_assert(BW_SMEM_BYTES <= 232448, "dK/dV kernel exceeds the opt-in shared memory");
// TMEM columns: S / P raw of buffer b at 64b, dP / dS raw at 64b + 32; their
// lo parts 128 further; the dV / dK accumulators of pair a at 256 + 128a
// (+ 64 for dK).
constexpr int BW_TMEM_COLS = 512;
constexpr uint32_t BW_IDESC_SD = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BW_NQ >> 3) << 17) |
                                 ((uint32_t)(QR >> 4) << 24);
constexpr uint32_t BW_IDESC_SD_BF = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BW_NQ >> 3) << 17) |
                                    ((uint32_t)(QR >> 4) << 24);   // bf16 x bf16 -> f32
constexpr uint32_t BW_IDESC_ACC = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                                  ((uint32_t)(QR >> 4) << 24);

struct BwArgs {
  const float *cosT, *sinT;   // RoPE table [T][HD/2]: the inverse rotation is applied to dK; nullptr: none
  const float *lse, *Drow;
  float *dsT, *dk, *dv;
  int B, H, KV;
  float scale;
  int *err;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// D (TMEM) (+)= A (TMEM, 128 lanes x 8 columns) * B (shared memory).
__device__ __forceinline__ void tc_mma_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p; }" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// lo = x - tf32(x) of n16 16-byte words at src, written at src + lo_off.
__device__ __forceinline__ void split_lo(uint8_t *src, int lo_off, int n16, int t, int nthreads) {
  for (int idx = t; idx < n16; idx += nthreads) {
    const float4 x = *reinterpret_cast<const float4 *>(src + idx * 16);
    float4 lo;
    lo.x = x.x - tf32_trunc(x.x); lo.y = x.y - tf32_trunc(x.y);
    lo.z = x.z - tf32_trunc(x.z); lo.w = x.w - tf32_trunc(x.w);
    *reinterpret_cast<float4 *>(src + lo_off + idx * 16) = lo;
  }
}


__global__ void __launch_bounds__(BW_THREADS, 1)
attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmKk, const __grid_constant__ CUtensorMap tmVk,
                        const __grid_constant__ CUtensorMap tmQk, const __grid_constant__ CUtensorMap tmOk,
                        const __grid_constant__ CUtensorMap tmQm, const __grid_constant__ CUtensorMap tmOm, BwArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + BW_DATA);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + BW_NBARS);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const uint32_t base = smem_u32(smem);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // [2]: one per raw buffer or TMEM buffer
  constexpr int KV_FULL = 0, KV_READY = 1, KM_FULL = 2, KM_READY = 4, KM_EMPTY = 5, MN_FULL = 7, MN_READY = 9,
                MN_EMPTY = 10, SD_FULL = 12, PD_READY = 14, ACC_FULL = 16, ACC_EMPTY = 18, FIN = 20;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbk = a.B * a.KV;
  const int kb = (int)blockIdx.x < nbk ? 0 : 1;          // the key blocks with 8 chunks per head first
  const int bk = (int)blockIdx.x % nbk, bb = bk / a.KV, kvh = bk % a.KV, grp = a.H / a.KV;
  const int c0 = 4 * kb, nc = T / BW_NQ - c0, n = grp * nc;
  const int key0 = QR * kb;

  if (threadIdx.x == 0) {
    mbar_init(bar(KV_FULL), 1);
    mbar_init(bar(KV_READY), 4);
    mbar_init(bar(KM_READY), 2);
    mbar_init(bar(MN_READY), 4);
    for (int x = 0; x < 2; x++) {
      mbar_init(bar(KM_FULL + x), 1);
      mbar_init(bar(KM_EMPTY + x), 1);
      mbar_init(bar(MN_FULL + x), 1);
      mbar_init(bar(MN_EMPTY + x), 1);
      mbar_init(bar(SD_FULL + x), 1);
      mbar_init(bar(PD_READY + x), 4);
      mbar_init(bar(ACC_FULL + x), 1);
      mbar_init(bar(ACC_EMPTY + x), 4);
    }
    mbar_init(bar(FIN), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BW_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ----------------------------------------------------------- producers
    if (lane < 2) {
      const bool mn = lane == 1;
      const CUtensorMap *mq = mn ? &tmQm : &tmQk, *mo = mn ? &tmOm : &tmOk;
      const int full = mn ? MN_FULL : KM_FULL, empty = mn ? MN_EMPTY : KM_EMPTY;
      const uint32_t raw = base + (mn ? BW_OFF_MNR : BW_OFF_KMR);
      if (!mn) {
        const int krow = bb * T + key0;
        mbar_arrive_expect_tx(bar(KV_FULL), 4 * BW_KTILE);
        for (int x = 0; x < 2; x++) {
          tma_load_2d(base + BW_OFF_K + x * BW_KTILE, &tmKk, bar(KV_FULL), kvh * HD + 32 * x, krow);
          tma_load_2d(base + BW_OFF_V + x * BW_KTILE, &tmVk, bar(KV_FULL), kvh * HD + 32 * x, krow);
        }
      }
      int issued = 0;
      for (int i = 0; i < n; i++) {
        const int r = i & 1, h = kvh * grp + i / nc, qrow = bb * T + BW_NQ * (c0 + i % nc);
        // Raw buffer r was last read by the products of chunk i - 2.
        if (i >= 2 && !mbar_wait(bar(empty + r), ((i - 2) >> 1) & 1, abort_flag, a.err, mn ? 62 : 61)) break;
        mbar_arrive_expect_tx(bar(full + r), BW_CBUF);
        const uint32_t dst = raw + r * BW_CBUF;
        for (int x = 0; x < 2; x++) {
          tma_load_2d(dst + x * BW_CTILE, mq, bar(full + r), h * HD + 32 * x, qrow);
          tma_load_2d(dst + BW_CB_O + x * BW_CTILE, mo, bar(full + r), h * HD + 32 * x, qrow);
        }
        issued = i + 1;
      }
      // No copy may still be landing when the CTA exits (phases of one
      // barrier complete in order, so the last one issued covers the rest).
      for (int i = issued > 2 ? issued - 2 : 0; i < issued; i++) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar(full + (i & 1)), (i >> 1) & 1)) {
          if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicExch(a.err, 63); break; }
        }
      }
      if (!mn) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar(KV_FULL), 0)) {
          if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicExch(a.err, 63); break; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      auto issue_sd = [&](int i) -> bool {
        const int b = i & 1;
        // TMEM buffer b was last read by the dV/dK products of chunk i - 2.
        if (i >= 2 && !mbar_wait(bar(MN_EMPTY + b), ((i - 2) >> 1) & 1, abort_flag, a.err, 64)) return false;
        if (!mbar_wait(bar(KM_READY), i & 1, abort_flag, a.err, 65)) return false;
        tc_fence_after();
        const uint32_t craw = base + BW_OFF_KMR + b * BW_CBUF, clo = base + BW_OFF_KML;
#pragma unroll
        for (int m = 0; m < 2; m++) {            // m = 0: S^T = K Q^T, 1: dP^T = V dO^T
          const uint32_t d = tmem + 64 * b + 32 * m;
          const uint32_t at = base + (m ? BW_OFF_V : BW_OFF_K), bo = m ? BW_CB_O : 0;
          // hi*hi: tf32 on the raw tiles
#pragma unroll
          for (int x = 0; x < 2; x++) {
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
              tc_mma(d, smem_desc(at + x * BW_KTILE + kk * 32, 16, 1024, LAYOUT_SW128),
                     smem_desc(craw + bo + x * BW_CTILE + kk * 32, 16, 1024, LAYOUT_SW128), BW_IDESC_SD,
                     (x > 0 || kk > 0) ? 1u : 0u);
          }
          // hi*lo + lo*hi: bf16 over the concatenated rows (two K = 16 steps
          // per 64-byte half)
#pragma unroll
          for (int x = 0; x < 2; x++) {
#pragma unroll
            for (int kc = 0; kc < 4; kc++) {
              const int off = (kc >> 1) * 64 + (kc & 1) * 32;
              tc_mma_bf16(d, smem_desc(at + BW_KV_LO + x * BW_KTILE + off, 16, 1024, LAYOUT_SW128),
                          smem_desc(clo + bo + x * BW_CTILE + off, 16, 1024, LAYOUT_SW128), BW_IDESC_SD_BF, 1);
            }
          }
        }
        tc_commit(bar(KM_EMPTY + b));
        tc_commit(bar(SD_FULL + b));
        return true;
      };
      auto issue_acc = [&](int i) -> bool {
        const int b = i & 1, g = i / nc, pa = g & 1;
        const bool first = i % nc == 0, last = i % nc == nc - 1;
        if (first && g >= 2 && !mbar_wait(bar(ACC_EMPTY + pa), ((g >> 1) - 1) & 1, abort_flag, a.err, 66))
          return false;
        if (!mbar_wait(bar(PD_READY + b), (i >> 1) & 1, abort_flag, a.err, 67)) return false;
        if (!mbar_wait(bar(MN_READY), i & 1, abort_flag, a.err, 68)) return false;
        tc_fence_after();
        const uint32_t craw = base + BW_OFF_MNR + b * BW_CBUF, clo = base + BW_OFF_MNL;
#pragma unroll
        for (int m = 0; m < 2; m++) {            // m = 0: dV += P^T dO, 1: dK += dS^T Q
          const uint32_t d = tmem + 256 + 128 * pa + 64 * m;
          const uint32_t a_hi = tmem + 64 * b + 32 * m, a_lo = a_hi + 128;
          const uint32_t bo = m ? 0 : BW_CB_O;
#pragma unroll
          for (int kk = 0; kk < BW_NQ / 8; kk++) {
            const uint64_t b_hi = smem_desc(craw + bo + kk * 1024, 4096, 512, LAYOUT_SW128_BASE32B);
            const uint64_t b_lo = smem_desc(clo + bo + kk * 1024, 4096, 512, LAYOUT_SW128_BASE32B);
            tc_mma_tmem_a(d, a_lo + kk * 8, b_hi, BW_IDESC_ACC, (!first || kk > 0) ? 1u : 0u);
            tc_mma_tmem_a(d, a_hi + kk * 8, b_lo, BW_IDESC_ACC, 1);
            tc_mma_tmem_a(d, a_hi + kk * 8, b_hi, BW_IDESC_ACC, 1);
          }
        }
        tc_commit(bar(MN_EMPTY + b));
        if (last) tc_commit(bar(ACC_FULL + pa));
        return true;
      };
      if (mbar_wait(bar(KV_READY), 0, abort_flag, a.err, 69) && issue_sd(0)) {
        for (int i = 0; i < n; i++) {
          if (i + 1 < n && !issue_sd(i + 1)) break;
          if (!issue_acc(i)) break;
        }
      }
      // Every issued MMA finished (also on the abort path) before TMEM is
      // read for the last time and released.
      tc_commit(bar(FIN));
      const long long t0 = clock64();
      while (!mbar_try_wait(bar(FIN), 0)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) { *abort_flag = 1; atomicExch(a.err, 70); break; }
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------ P^T and dS^T (a key row each)
    const int q4 = warp & 3, row = q4 * 32 + lane, key = key0 + row;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    // The chunk's 32 lse and D values, one per lane, loaded a chunk ahead and
    // broadcast by shuffles.
    auto chunk_row = [&](int i) { return ((size_t)bb * a.H + kvh * grp + i / nc) * T + BW_NQ * (c0 + i % nc); };
    // P = exp(scale s - lse) = 2^(s scale log2(e) - lse log2(e)); lse is kept
    // pre-multiplied by log2(e).
    const float c2 = a.scale * 1.4426950408889634f;
    float l_nx = __ldg(a.lse + chunk_row(0) + lane) * 1.4426950408889634f, d_nx = __ldg(a.Drow + chunk_row(0) + lane);
    for (int i = 0; i < n; i++) {
      const int b = i & 1, q0 = BW_NQ * (c0 + i % nc);
      const size_t crow = chunk_row(i);
      const float l_me = l_nx, d_me = d_nx;
      if (i + 1 < n) {
        l_nx = __ldg(a.lse + chunk_row(i + 1) + lane) * 1.4426950408889634f;
        d_nx = __ldg(a.Drow + chunk_row(i + 1) + lane);
      }
      if (!__all_sync(0xffffffffu, mbar_wait(bar(SD_FULL + b), (i >> 1) & 1, abort_flag, a.err, 71))) break;
      tc_fence_after();
      uint32_t sv[32], dv[32];
      tmem_ld32(tmem + lane_addr + 64 * b, sv);
      tmem_ld32(tmem + lane_addr + 64 * b + 32, dv);
      // P and dS; lo parts through one buffer.
      float ph[32], dh[32], lo[32];
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const float ls = __shfl_sync(0xffffffffu, l_me, e), ds = __shfl_sync(0xffffffffu, d_me, e);
        const float pr = key <= q0 + e ? exp2f(fmaf(__uint_as_float(sv[e]), c2, -ls)) : 0.0f;
        ph[e] = pr;
        dh[e] = pr * (__uint_as_float(dv[e]) - ds) * a.scale;
      }
      tmem_st32(tmem + lane_addr + 64 * b, ph);
      tmem_st32(tmem + lane_addr + 64 * b + 32, dh);
#pragma unroll
      for (int e = 0; e < 32; e++) lo[e] = ph[e] - tf32_trunc(ph[e]);
      tmem_st32(tmem + lane_addr + 128 + 64 * b, lo);
#pragma unroll
      for (int e = 0; e < 32; e++) lo[e] = dh[e] - tf32_trunc(dh[e]);
      tmem_st32(tmem + lane_addr + 128 + 64 * b + 32, lo);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(PD_READY + b));
      // crow = (bh * T + q0): the scratch row of this key is bh * T + key.
      float4 *dst = reinterpret_cast<float4 *>(a.dsT + (crow - q0 + key) * T + q0);
#pragma unroll
      for (int e = 0; e < 32; e += 4) dst[e / 4] = make_float4(dh[e], dh[e + 1], dh[e + 2], dh[e + 3]);
    }
  } else if (warp >= 10) {
    // ----------------------------------- bf16 halves of the K-major tiles
    const int t = threadIdx.x - 320;             // 0..63
    for (int i = 0; i < n; i++) {
      const int r = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(KM_FULL + r), (i >> 1) & 1, abort_flag, a.err, 74))) break;
      // The lo buffer is free once the previous chunk's S^T / dP^T are done.
      if (i >= 1 && !__all_sync(0xffffffffu, mbar_wait(bar(KM_EMPTY + (r ^ 1)), ((i - 1) >> 1) & 1, abort_flag,
                                                        a.err, 76)))
        break;
      split_cat(smem + BW_OFF_KMR + r * BW_CBUF, smem + BW_OFF_KML, BW_CBUF / 128, true, t, 64);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(KM_READY));
    }
  } else {
    // ------- lo parts of K, V and the MN-major tiles; dV / dK per head
    const int t = threadIdx.x - 192, q4 = warp & 3, row = q4 * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    float accv[HD], acck[HD];
#pragma unroll
    for (int e = 0; e < HD; e++) { accv[e] = 0.0f; acck[e] = 0.0f; }
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar(KV_FULL), 0, abort_flag, a.err, 72));
    if (ok) {
      split_cat(smem + BW_OFF_K, smem + BW_OFF_K + BW_KV_LO, 2 * BW_KTILE / 128, false, t, 128);
      split_cat(smem + BW_OFF_V, smem + BW_OFF_V + BW_KV_LO, 2 * BW_KTILE / 128, false, t, 128);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(KV_READY));
    }
    auto drain = [&](int g) -> bool {
      const int pa = g & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(ACC_FULL + pa), (g >> 1) & 1, abort_flag, a.err, 73))) return false;
      tc_fence_after();
#pragma unroll
      for (int m = 0; m < 2; m++) {
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
          uint32_t v[16];
          tmem_ld16(tmem + lane_addr + 256 + 128 * pa + 64 * m + 16 * cc, v);
#pragma unroll
          for (int e = 0; e < 16; e++) {
            if (m == 0) accv[16 * cc + e] += __uint_as_float(v[e]);
            else acck[16 * cc + e] += __uint_as_float(v[e]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ACC_EMPTY + pa));
      return true;
    };
    for (int i = 0; i < n && ok; i++) {
      const int r = i & 1;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(bar(MN_FULL + r), (i >> 1) & 1, abort_flag, a.err, 75)))) break;
      // The lo buffer is free once the previous chunk's dV / dK are done.
      if (i >= 1 && !(ok = __all_sync(0xffffffffu, mbar_wait(bar(MN_EMPTY + (r ^ 1)), ((i - 1) >> 1) & 1,
                                                              abort_flag, a.err, 77))))
        break;
      split_lo(smem + BW_OFF_MNR + r * BW_CBUF, BW_OFF_MNL - (BW_OFF_MNR + r * BW_CBUF), BW_CBUF / 16, t, 128);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(MN_READY));
      // The previous head's accumulators (its last products are done: the
      // lo buffer wait above covered them).
      if (i > 0 && (i - 1) % nc == nc - 1) ok = drain((i - 1) / nc);
    }
    if (ok) ok = drain(grp - 1);
    if (ok && !*abort_flag) {
      const size_t o = ((size_t)bb * T + key0 + row) * (size_t)(a.KV * HD) + (size_t)kvh * HD;
      if (a.cosT)
        rope_back_row(acck, a.cosT + (size_t)(key0 + row) * (HD / 2), a.sinT + (size_t)(key0 + row) * (HD / 2));
      float4 *pv = reinterpret_cast<float4 *>(a.dv + o);
      float4 *pk = reinterpret_cast<float4 *>(a.dk + o);
#pragma unroll
      for (int e = 0; e < HD; e += 4) {
        pv[e / 4] = make_float4(accv[e], accv[e + 1], accv[e + 2], accv[e + 3]);
        pk[e / 4] = make_float4(acck[e], acck[e + 1], acck[e + 2], acck[e + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BW_TMEM_COLS) : "memory");
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;

static int map2d(CUtensorMap *m, const float *p, uint64_t inner, uint64_t outer, uint32_t bx, uint32_t by,
                 CUtensorMapSwizzle sw) {
  if (!g_enc) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return set_error(TL_ECUDA, "cuTensorMapEncodeTiled not available from the driver");
    g_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint64_t dims[2] = {inner, outer}, strides[1] = {inner * 4};
  cuuint32_t box[2] = {bx, by}, es[2] = {1, 1};
  CUresult r = g_enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(p), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TL_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TL_OK;
}

}  // namespace atc

// True when the tensor-core forward takes this shape.
bool attn_fwd_tc_supported(const float *q, const float *k, const float *v, int T, int hd, int H, int KV) {
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v);
  return T == atc::T && hd == atc::HD && (al & 15) == 0 && KV > 0 && H % KV == 0;
}

int attn_fwd_tc(DeviceCtx *c, const float *q, const float *k, const float *v, float *out, float *lse, int B, int T,
                int H, int KV, int hd) {
  (void)T;
  (void)hd;
  static bool attr[kMaxDevices] = {};
  if (!attr[c->device]) {
    TL_TRY_CUDA(cudaFuncSetAttribute(atc::attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     atc::SMEM_BYTES));
    attr[c->device] = true;
  }
  const int D = H * atc::HD, KD = KV * atc::HD;
  const uint64_t rows = (uint64_t)B * atc::T;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = atc::map2d(&mq, q, D, rows, 32, atc::QR, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = atc::map2d(&mk, k, KD, rows, 32, atc::QR, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = atc::map2d(&mv, v, KD, rows, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))) return rc;
  atc::Args a;
  a.out = out; a.lse = lse; a.H = H; a.KV = KV; a.D = D;
  a.items = B * H;
  a.scale = 1.0f / sqrtf((float)atc::HD);
  a.err = c->err_flag;
  // One pair per SM pair, each walking its share of the items.  Tests cap the
  // pair count (TL_ATTN_FWD_PAIRS) to give each pair long item chains at small
  // batch sizes.
  int npairs = std::min(a.items, std::max(1, c->num_sms / 2));
  if (const char *e = getenv("TL_ATTN_FWD_PAIRS")) {
    const int cap = atoi(e);
    if (cap > 0 && cap < npairs) npairs = cap;
  }
  TraceScope ts(c, "k_attn_fwd_tc");
  atc::attn_fwd_tc_kernel<<<2 * npairs, atc::NUM_THREADS, atc::SMEM_BYTES, c->stream>>>(mq, mk, mv, a);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

// True when the tensor-core dQ product takes this shape (the forward's).
bool attn_bwd_dq_tc_supported(const float *dsT, const float *k, const float *dq, int T, int hd, int H, int KV) {
  const uintptr_t al =
      reinterpret_cast<uintptr_t>(dsT) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(dq);
  return T == atc::T && hd == atc::HD && (al & 15) == 0 && KV > 0 && H % KV == 0;
}

int attn_bwd_dq_tc(DeviceCtx *c, const float *dsT, const float *k, float *dq, int B, int H, int KV, const float *cosT,
                   const float *sinT) {
  static bool attr[kMaxDevices] = {};
  if (!attr[c->device]) {
    TL_TRY_CUDA(cudaFuncSetAttribute(atc::attn_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     atc::DQ_SMEM_BYTES));
    attr[c->device] = true;
  }
  const int KD = KV * atc::HD;
  CUtensorMap ms, mk;
  int rc;
  if ((rc = atc::map2d(&ms, dsT, atc::T, (uint64_t)B * H * atc::T, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)))
    return rc;
  if ((rc = atc::map2d(&mk, k, KD, (uint64_t)B * atc::T, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))) return rc;
  atc::DqArgs a;
  a.dq = dq; a.cosT = cosT; a.sinT = sinT; a.B = B; a.H = H; a.KV = KV; a.D = H * atc::HD; a.err = c->err_flag;
  // persistent: one CTA per SM (or per item, when there are fewer)
  const int grid = std::min(2 * B * H, std::max(1, c->num_sms));
  TraceScope ts(c, "k_attn_bwd_dq_tc");
  atc::attn_bwd_dq_tc_kernel<<<grid, atc::DQ_THREADS, atc::DQ_SMEM_BYTES, c->stream>>>(ms, mk, a);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

// True when the tensor-core dK/dV kernel takes this shape (the forward's).
bool attn_bwd_dkdv_tc_supported(const float *const *ptrs, int nptr, int T, int hd, int H, int KV) {
  uintptr_t al = 0;
  for (int i = 0; i < nptr; i++) al |= reinterpret_cast<uintptr_t>(ptrs[i]);
  return T == atc::T && hd == atc::HD && (al & 15) == 0 && KV > 0 && H % KV == 0;
}

int attn_bwd_dkdv_tc(DeviceCtx *c, const float *q, const float *k, const float *v, const float *dout,
                     const float *lse, const float *Drow, float *dsT, float *dk, float *dv, int B, int H, int KV,
                     const float *cosT, const float *sinT) {
  static bool attr[kMaxDevices] = {};
  if (!attr[c->device]) {
    TL_TRY_CUDA(cudaFuncSetAttribute(atc::attn_bwd_dkdv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     atc::BW_SMEM_BYTES));
    attr[c->device] = true;
  }
  const int D = H * atc::HD, KD = KV * atc::HD;
  const uint64_t rows = (uint64_t)B * atc::T;
  CUtensorMap mkk, mvk, mqk, mok, mqm, mom;
  int rc;
  if ((rc = atc::map2d(&mkk, k, KD, rows, 32, atc::QR, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = atc::map2d(&mvk, v, KD, rows, 32, atc::QR, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = atc::map2d(&mqk, q, D, rows, 32, atc::BW_NQ, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = atc::map2d(&mok, dout, D, rows, 32, atc::BW_NQ, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  if ((rc = atc::map2d(&mqm, q, D, rows, 32, atc::BW_NQ, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))) return rc;
  if ((rc = atc::map2d(&mom, dout, D, rows, 32, atc::BW_NQ, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))) return rc;
  atc::BwArgs a;
  a.cosT = cosT; a.sinT = sinT;
  a.lse = lse; a.Drow = Drow; a.dsT = dsT; a.dk = dk; a.dv = dv;
  a.B = B; a.H = H; a.KV = KV;
  a.scale = 1.0f / sqrtf((float)atc::HD);
  a.err = c->err_flag;
  TraceScope ts(c, "k_attn_bwd_dkdv_tc");
  atc::attn_bwd_dkdv_tc_kernel<<<2 * B * KV, atc::BW_THREADS, atc::BW_SMEM_BYTES, c->stream>>>(mkk, mvk, mqk, mok,
                                                                                               mqm, mom, a);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

int attn_tc_prepare(DeviceCtx *c) {
  TL_TRY_CUDA(cudaFuncSetAttribute(atc::attn_bwd_dkdv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   atc::BW_SMEM_BYTES));
  TL_TRY_CUDA(cudaFuncSetAttribute(atc::attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   atc::SMEM_BYTES));
  TL_TRY_CUDA(cudaFuncSetAttribute(atc::attn_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   atc::DQ_SMEM_BYTES));
  (void)c;
  return TL_OK;
}

}  // namespace tl
