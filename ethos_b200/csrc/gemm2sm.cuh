// Persistent 2-SM tcgen05 GEMM  D[M, N] = sum_k A[m, k] * B[n, k]  (bf16 in,
// fp32 TMEM accumulate) with the operand majors, split-K and per-row
// epilogues of gemm.cuh.
//
// A cluster of two CTAs (one SM pair) owns a 256 x 256 output tile: CTA r
// stages rows [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128)
// of the B tile, and the leader's tcgen05.mma.cta_group::2 (M = 256, N = 256,
// K = 16) reads both CTAs' shared memory, so each SM holds half of B and
// receives 32 KB of operands per 64-deep K block for 128 x 256 x 64 MACs,
// two thirds of the single-SM kernel's 48 KB.  CTA r's TMEM holds rows
// [128 r, 128 r + 128) of the tile (all 256 columns), read by its own
// epilogue warps.  No load uses cluster multicast; only the MMA completion
// (tcgen05.commit) is multicast to both CTAs.
//
// Barriers (all in the CTA's own shared memory):
//   full[s]      leader only: one arrive.expect_tx (both CTAs' bytes) plus
//                the complete_tx of both CTAs' copies.
//   empty[s]     both CTAs: the leader's commit, multicast.
//   acc_full[b]  both CTAs: the leader's commit, multicast.
//   acc_empty[b] leader only: one arrive per epilogue warp of both CTAs
//                (the peer's arrive remotely through its cluster address).
// Roles per CTA: warp 0 = TMA producer, warp 1 = TMEM owner (+ MMA issuer in
// the leader), warps 2.. = epilogue.  Every wait is bounded (mbar_wait); the
// CTAs meet at cluster barriers after set-up and before TMEM is freed.
#pragma once

#include "gemm.cuh"

namespace ethos {

constexpr int G2_BM = 128;  // rows per CTA (tile M = 256)
constexpr int G2_BN = 256;  // tile N (each CTA stages 128 rows of B)
constexpr int G2_BK = 64;
constexpr int G2_STAGES = 6;
constexpr int G2_A_BYTES = G2_BM * G2_BK * 2;
constexpr int G2_B_BYTES = (G2_BN / 2) * G2_BK * 2;
constexpr int G2_STAGE_BYTES = G2_A_BYTES + G2_B_BYTES;

struct Gemm2Ctl {
  uint64_t full[G2_STAGES];
  uint64_t empty[G2_STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <class Epi>
struct Gemm2Cfg {
  static constexpr int kEpiWarps = Epi::kEpiWarps;
  static_assert(kEpiWarps == 8 || kEpiWarps == 16, "8 or 16 epilogue warps");
  static constexpr int kEpiThreads = 32 * kEpiWarps;
  static constexpr int kThreads = 64 + kEpiThreads;
  static constexpr int kSmem = G2_STAGES * G2_STAGE_BYTES + GEMM_COLP_BYTES + kEpiWarps * GEMM_STG_WARP_BYTES + 1024 +
                               static_cast<int>(sizeof(Gemm2Ctl));
  static_assert(kSmem <= 227 * 1024, "2-SM GEMM shared memory");
  static_assert(!Epi::kTmaStore, "TMA-store epilogues run on the single-SM kernel");
};

// ------------------------------------------------------ cluster helpers --
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address in the cluster shared window of `smem_addr` (a shared::cta
// address of this CTA) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2-D tile load into this CTA's shared memory whose completion is counted on
// the barrier at `bar_cluster` (the leader's full barrier; cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* tm, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at the same offset in every CTA of `mask` when
// the pair's previously issued MMAs have completed.
__device__ __forceinline__ void umma_commit_pair_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- kernel --
// Launched with cluster dimension (2, 1, 1); work unit u (tile u % tiles of
// ceil(M/256) x N/256, K slice u / tiles) is owned by cluster u mod
// (gridDim.x / 2) in turn.  MN-major operands are staged as two 64-wide
// boxes per CTA (LBO 8 KB), as in k_gemm.
template <class Epi, bool kAMN, bool kBMN>
__global__ void __launch_bounds__(Gemm2Cfg<Epi>::kThreads, 1)
    k_gemm2sm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
              int ksplit, Epi epi, int* err) {
  using Cfg = Gemm2Cfg<Epi>;
  constexpr int CHUNKS = (G2_BN / 32) / (Cfg::kEpiWarps / 4);  // 32-column chunks per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* colp_s = smem + G2_STAGES * G2_STAGE_BYTES;
  uint8_t* stg_s = colp_s + GEMM_COLP_BYTES;
  Gemm2Ctl* ctl = reinterpret_cast<Gemm2Ctl*>(stg_s + Cfg::kEpiWarps * GEMM_STG_WARP_BYTES);
  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) >> 1;
  const int num_pairs = static_cast<int>(gridDim.x) >> 1;
  const int num_n = N / G2_BN;
  const int num_tiles = ((M + 2 * G2_BM - 1) / (2 * G2_BM)) * num_n;
  const int num_kb = (K + G2_BK - 1) / G2_BK;
  const int kpb = (num_kb + ksplit - 1) / ksplit;  // K blocks per split (host guarantees none is empty)
  const int num_units = num_tiles * ksplit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < G2_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], 2 * Cfg::kEpiWarps);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, 2 * G2_BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote arrive or commit
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  pdl_launch_dependents();
  pdl_wait();  // set-up above touched only shared memory, TMEM and parameters
  volatile int* abort = &ctl->abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      RingPos rp;
      bool ok = true;
      for (int u = pair; ok && u < num_units; u += num_pairs) {
        const int tile = u % num_tiles;
        const int ks = u / num_tiles;
        const int m0 = (tile / num_n) * (2 * G2_BM) + static_cast<int>(rank) * G2_BM;
        const int n0 = (tile % num_n) * G2_BN + static_cast<int>(rank) * (G2_BN / 2);
        const int kb1 = min(num_kb, (ks + 1) * kpb);
        for (int kb = ks * kpb; kb < kb1; ++kb) {
          if (!mbar_wait(&ctl->empty[rp.stage], rp.phase ^ 1u, abort, err, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + rp.stage * G2_STAGE_BYTES;
          uint8_t* sb = sa + G2_A_BYTES;
          if (leader) mbar_arrive_expect_tx(&ctl->full[rp.stage], 2 * G2_STAGE_BYTES);
          const uint32_t fb = cluster_map(smem_u32(&ctl->full[rp.stage]), 0);
          if (kAMN) {
            tma_load_2d_pair(sa, &tmA, fb, m0, kb * G2_BK);
            tma_load_2d_pair(sa + 8192, &tmA, fb, m0 + 64, kb * G2_BK);
          } else {
            tma_load_2d_pair(sa, &tmA, fb, kb * G2_BK, m0);
          }
          if (kBMN) {
            tma_load_2d_pair(sb, &tmB, fb, n0, kb * G2_BK);
            tma_load_2d_pair(sb + 8192, &tmB, fb, n0 + 64, kb * G2_BK);
          } else {
            tma_load_2d_pair(sb, &tmB, fb, kb * G2_BK, n0);
          }
          rp.advance(G2_STAGES);
        }
      }
      if (!ok) {
        // Copies still in flight must land before the CTA's shared memory
        // goes away.  Both CTAs' copies complete on the leader's full
        // barriers: the leader waits for the phases of its most recent
        // stages (bounded waits); the peer, which cannot see those barriers,
        // waits a bounded 100 us, far above the latency of a 16 KB copy.
        if (leader) {
          rp.drain(ctl->full, G2_STAGES, err, 5);
        } else {
          const uint64_t t0 = global_timer_ns();
          while (global_timer_ns() - t0 < 100000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = umma_idesc_bf16_f32_major(2 * G2_BM, G2_BN, kAMN, kBMN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = pair; ok && u < num_units; u += num_pairs, ++it) {
        const int ks = u / num_tiles;
        const int kb0 = ks * kpb, kb1 = min(num_kb, (ks + 1) * kpb);
        const int buf = it & 1;
        const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
        if (!mbar_wait(&ctl->acc_empty[buf], acc_phase ^ 1u, abort, err, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * G2_BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&ctl->full[stage], phase, abort, err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * G2_STAGE_BYTES);
          const uint32_t b_base = a_base + G2_A_BYTES;
#pragma unroll
          for (int k = 0; k < G2_BK / 16; ++k) {
            const uint64_t ad = kAMN ? umma_desc_sw128_mn(a_base + k * 2048, 8192) : umma_desc_sw128(a_base + k * 32);
            const uint64_t bd = kBMN ? umma_desc_sw128_mn(b_base + k * 2048, 8192) : umma_desc_sw128(b_base + k * 32);
            umma_bf16_pair(d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair_mc(&ctl->empty[stage], 0x3);
          if (++stage == G2_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(&ctl->acc_full[buf], 0x3);
      }
      if (!ok || *abort) {
        // Drain: wait until every MMA of the pair has completed.
        umma_commit_pair(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr, err, 6);
      }
    }
  } else {
    // Epilogue warps never leave the tile loop early: after an abort they skip
    // the work but still take every named barrier and arrive on every
    // acc_empty phase, so no partner can block.
    const int q = warp & 3;
    const int ch = (warp - 2) >> 2;  // column group of the tile (CHUNKS chunks each)
    const uint32_t acc_empty_leader0 = cluster_map(smem_u32(&ctl->acc_empty[0]), 0);
    const uint32_t acc_empty_leader1 = cluster_map(smem_u32(&ctl->acc_empty[1]), 0);
    int it = 0;
    bool ok = true;
    for (int u = pair; u < num_units; u += num_pairs, ++it) {
      const int tile = u % num_tiles;
      const int buf = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
      const int m0 = (tile / num_n) * (2 * G2_BM) + static_cast<int>(rank) * G2_BM;
      const int n0 = (tile % num_n) * G2_BN;
      uint8_t* cps = colp_s + buf * 256 * 8;
      if (Epi::kColParamBytes > 0) {
        // stage this tile's column data (its previous user, tile it-2, was
        // released by the barrier of tile it-1)
        const int tid = static_cast<int>(threadIdx.x) - 64;
        if (tid < 256) epi.load_col_params(n0, cps, tid);
        named_bar_sync(1, Cfg::kEpiThreads);
      }
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&ctl->acc_full[buf], acc_phase, abort, err, 4));
      if (ok) {
        tc_fence_after();
        const int row = m0 + q * 32 + lane;
        EpiCtx cx{stg_s + (warp - 2) * GEMM_STG_WARP_BYTES, m0 + q * 32, min(32, M - (m0 + q * 32)), lane, 0};
#pragma unroll 1
        for (int c = ch * CHUNKS; c < (ch + 1) * CHUNKS; ++c) {
          float v[32];
          tmem_ld32(tmem_addr(tmem, q * 32, buf * G2_BN + c * 32), v);
          cx.chunk = c - ch * CHUNKS;
          epi(row, n0 + c * 32, v, cps, cx);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(buf ? acc_empty_leader1 : acc_empty_leader0);
    }
  }

  // Teardown: every accumulator was consumed (or the roles gave up and the
  // leader drained its MMAs); the peer's shared memory and barriers stay
  // alive until both CTAs arrive here.
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * G2_BN);
  }
}

}  // namespace ethos
