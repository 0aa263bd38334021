// Product-key router kernels: sub-key scoring on tcgen05 with a fused top-k
// epilogue (per-half top-k, candidate-grid top-k, fp32 softmax, id decode),
// and the BatchNorm batch-statistics / normalisation kernels of training mode.
//
// Reference: ProductKeyRouter.forward, model.py:208-254.
#pragma once

#include <cfloat>

#include "gemm.cuh"

namespace ethos {

// ----------------------------------------------------------- top-k lists --
// Branch-free sorted-descending insertion into a register list of N entries.
// A score not above the last entry (or -inf) leaves the list unchanged; strict
// '>' keeps the earlier of two equal scores first.
template <int N>
__device__ __forceinline__ void topk_insert(float (&v)[N], int (&ix)[N], float s, int id) {
  bool c[N];
#pragma unroll
  for (int j = 0; j < N; ++j) c[j] = s > v[j];
#pragma unroll
  for (int j = N - 1; j > 0; --j) {
    v[j] = c[j - 1] ? v[j - 1] : (c[j] ? s : v[j]);
    ix[j] = c[j - 1] ? ix[j - 1] : (c[j] ? id : ix[j]);
  }
  v[0] = c[0] ? s : v[0];
  ix[0] = c[0] ? id : ix[0];
}

// Folds 32 scores of this lane's row (s[i] for key key0 + i) into the list,
// considering only scores >= tau.  Candidates (>= tau and above the current
// N-th best) are marked in a bitmask and inserted in a warp-uniform loop that
// runs max-over-lanes(#candidates) times; the chunk is staged in this warp's
// shared buffer `stage` ([i][lane] layout, conflict-free) so each lane can
// fetch its i-th candidate.
template <int N, bool kExplicitIds>
__device__ __forceinline__ void topk_fold_chunk(float (&v)[N], int (&ix)[N], const float (&s)[32], const int* id,
                                                int key0, float tau, float* stage, int* stage_id, int lane) {
  const float thr = v[N - 1];
  uint32_t mask = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) mask |= ((s[i] >= tau && s[i] > thr) ? 1u : 0u) << i;
  if (!__any_sync(0xffffffffu, mask != 0u)) return;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    stage[i * 32 + lane] = s[i];
    if (kExplicitIds) stage_id[i * 32 + lane] = id[i];
  }
  __syncwarp();
  while (__any_sync(0xffffffffu, mask != 0u)) {
    const int i = mask ? __ffs(mask) - 1 : 0;
    const float sv = mask ? stage[i * 32 + lane] : -INFINITY;
    const int si = kExplicitIds ? stage_id[i * 32 + lane] : key0 + i;
    mask &= mask - 1u;
    topk_insert<N>(v, ix, sv, si);
  }
  __syncwarp();
}

// Sorts a[0..N) descending (N a power of two) with a bitonic network of
// min/max exchanges.
template <int N>
__device__ __forceinline__ void bitonic_sort_desc(float (&a)[N]) {
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const bool desc = (i & k) == 0;
          const float x = a[i], y = a[l];
          a[i] = desc ? fmaxf(x, y) : fminf(x, y);
          a[l] = desc ? fminf(x, y) : fmaxf(x, y);
        }
      }
    }
  }
}

// Sorting networks over (score, id) pairs in registers: fixed, branch-free
// compare-exchange sequences with eight or more independent exchanges per
// stage.  ce_desc leaves the larger score at (a, ia); equal scores keep their
// places.
__device__ __forceinline__ void ce_desc(float& a, int& ia, float& b, int& ib) {
  const bool sw = b > a;
  const float va = sw ? b : a, vb = sw ? a : b;
  const int ja = sw ? ib : ia, jb = sw ? ia : ib;
  a = va;
  b = vb;
  ia = ja;
  ib = jb;
}
// bitonic sequence -> sorted descending
template <int N>
__device__ __forceinline__ void bitonic_merge_desc_kv(float (&v)[N], int (&ix)[N]) {
#pragma unroll
  for (int j = N >> 1; j > 0; j >>= 1) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if ((i & j) == 0) ce_desc(v[i], ix[i], v[i | j], ix[i | j]);
    }
  }
}
// (a, ia) <- the N largest of a and b (both sorted descending), sorted:
// max(a[i], b[N-1-i]) is bitonic and holds the top N of the union.
template <int N>
__device__ __forceinline__ void top_merge_kv(float (&a)[N], int (&ia)[N], const float (&b)[N], const int (&ib)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const bool tb = b[N - 1 - i] > a[i];
    a[i] = tb ? b[N - 1 - i] : a[i];
    ia[i] = tb ? ib[N - 1 - i] : ia[i];
  }
  bitonic_merge_desc_kv<N>(a, ia);
}
// out <- a ++ b sorted descending (a, b sorted descending)
template <int N>
__device__ __forceinline__ void merge_sorted_kv(const float (&a)[N], const int (&ia)[N], const float (&b)[N],
                                                const int (&ib)[N], float (&out)[2 * N], int (&oi)[2 * N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    out[i] = a[i];
    oi[i] = ia[i];
    out[N + i] = b[N - 1 - i];
    oi[N + i] = ib[N - 1 - i];
  }
  bitonic_merge_desc_kv<2 * N>(out, oi);
}
// Row i of the candidate grid: a[i] + b[j] for j < n (padded with -inf to P).
template <int P, int TOPK>
__device__ __forceinline__ void grid_row(const float (&a)[TOPK], const int (&ia)[TOPK], const float (&b)[TOPK],
                                         const int (&ib)[TOPK], int i, int n, int K, float (&v)[P], int (&ix)[P]) {
#pragma unroll
  for (int j = 0; j < P; ++j) {
    v[j] = j < n ? a[i] + b[j] : -INFINITY;
    ix[j] = j < n ? ia[i] * K + ib[j] : 0;
  }
}
// Top TOPK of the grid a[i] + b[j] (a, b sorted descending), sorted.  Only
// pairs with (i+1)(j+1) <= TOPK can rank in the top TOPK (every (i', j') with
// i' <= i, j' <= j scores at least as high), so row i has TOPK/(i+1) entries;
// the rows are sorted and are merged by networks.
template <int TOPK>
__device__ __forceinline__ void grid_topk(const float (&a)[TOPK], const int (&ia)[TOPK], const float (&b)[TOPK],
                                          const int (&ib)[TOPK], int K, float (&f)[TOPK], int (&fi)[TOPK]) {
  grid_row<TOPK, TOPK>(a, ia, b, ib, 0, TOPK, K, f, fi);
  if constexpr (TOPK == 16) {
    // rows 1 (8 entries) + the singles a[8..15] + b[0]
    {
      float r1[8], z[8], w[16];
      int j1[8], jz[8], jw[16];
      grid_row<8, 16>(a, ia, b, ib, 1, 8, K, r1, j1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        z[i] = a[8 + i] + b[0];
        jz[i] = ia[8 + i] * K + ib[0];
      }
      merge_sorted_kv<8>(r1, j1, z, jz, w, jw);
      top_merge_kv<16>(f, fi, w, jw);
    }
    // rows 2 (5) and 3 (4)
    {
      float r2[8], r3[8], x[16];
      int j2[8], j3[8], jx[16];
      grid_row<8, 16>(a, ia, b, ib, 2, 5, K, r2, j2);
      grid_row<8, 16>(a, ia, b, ib, 3, 4, K, r3, j3);
      merge_sorted_kv<8>(r2, j2, r3, j3, x, jx);
      top_merge_kv<16>(f, fi, x, jx);
    }
    // rows 4..7 (3, 2, 2, 2)
    {
      float r4[4], r5[4], r6[4], r7[4], y1[8], y2[8], y[16];
      int j4[4], j5[4], j6[4], j7[4], k1[8], k2[8], jy[16];
      grid_row<4, 16>(a, ia, b, ib, 4, 3, K, r4, j4);
      grid_row<4, 16>(a, ia, b, ib, 5, 2, K, r5, j5);
      grid_row<4, 16>(a, ia, b, ib, 6, 2, K, r6, j6);
      grid_row<4, 16>(a, ia, b, ib, 7, 2, K, r7, j7);
      merge_sorted_kv<4>(r4, j4, r5, j5, y1, k1);
      merge_sorted_kv<4>(r6, j6, r7, j7, y2, k2);
      merge_sorted_kv<8>(y1, k1, y2, k2, y, jy);
      top_merge_kv<16>(f, fi, y, jy);
    }
  } else {
#pragma unroll
    for (int i = 1; i < TOPK; ++i) {
      float r[TOPK];
      int jr[TOPK];
      grid_row<TOPK, TOPK>(a, ia, b, ib, i, TOPK / (i + 1), K, r, jr);
      top_merge_kv<TOPK>(f, fi, r, jr);
    }
  }
}

// The TOPK = 16 grid merge tree in two independent parts: rows 0 and 1 with
// the singles a[8..15] + b[0], and rows 2..7; the top 16 of the two results
// is the grid's top 16 (the same rows as grid_topk<16>).
template <int TOPK>
__device__ __forceinline__ void grid_rows01(const float (&a)[TOPK], const int (&ia)[TOPK], const float (&b)[TOPK],
                                            const int (&ib)[TOPK], int K, float (&f)[TOPK], int (&fi)[TOPK]) {
  static_assert(TOPK == 16, "split tree is for top 16");
  grid_row<16, 16>(a, ia, b, ib, 0, 16, K, f, fi);
  float r1[8], z[8], w[16];
  int j1[8], jz[8], jw[16];
  grid_row<8, 16>(a, ia, b, ib, 1, 8, K, r1, j1);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    z[i] = a[8 + i] + b[0];
    jz[i] = ia[8 + i] * K + ib[0];
  }
  merge_sorted_kv<8>(r1, j1, z, jz, w, jw);
  top_merge_kv<16>(f, fi, w, jw);
}
template <int TOPK>
__device__ __forceinline__ void grid_rows27(const float (&a)[TOPK], const int (&ia)[TOPK], const float (&b)[TOPK],
                                            const int (&ib)[TOPK], int K, float (&f)[TOPK], int (&fi)[TOPK]) {
  static_assert(TOPK == 16, "split tree is for top 16");
  float r2[8], r3[8];
  int j2[8], j3[8];
  grid_row<8, 16>(a, ia, b, ib, 2, 5, K, r2, j2);
  grid_row<8, 16>(a, ia, b, ib, 3, 4, K, r3, j3);
  merge_sorted_kv<8>(r2, j2, r3, j3, f, fi);
  float r4[4], r5[4], r6[4], r7[4], y1[8], y2[8], y[16];
  int j4[4], j5[4], j6[4], j7[4], k1[8], k2[8], jy[16];
  grid_row<4, 16>(a, ia, b, ib, 4, 3, K, r4, j4);
  grid_row<4, 16>(a, ia, b, ib, 5, 2, K, r5, j5);
  grid_row<4, 16>(a, ia, b, ib, 6, 2, K, r6, j6);
  grid_row<4, 16>(a, ia, b, ib, 7, 2, K, r7, j7);
  merge_sorted_kv<4>(r4, j4, r5, j5, y1, k1);
  merge_sorted_kv<4>(r6, j6, r7, j7, y2, k2);
  merge_sorted_kv<8>(y1, k1, y2, k2, y, jy);
  top_merge_kv<16>(f, fi, y, jy);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ------------------------------------------------------ scoring + top-k --
// One work item = (head h, tile of 128 tokens); per item two halves p, per
// half the sub-keys in units of up to 256 (TMEM buffer = unit parity, so the
// two units of a 512-key half fill all 512 columns).
// The MMA warp computes S[t, key] = sum_c A[t, c] * B[key, c] into the
// unit's 256-column TMEM buffer; 8 epilogue warps (one token row per thread)
// in two groups, group g taking columns [128 g, 128 g + 128) of every unit,
// select the half's top-k per row exactly:
//   1. maxima of the 8-key groups (three-input max), top 16 per group;
//   2. tau = k-th largest of the half's 64 maxima (the groups' sorted lists
//      exchanged through shared memory): a lower bound on the half's k-th
//      largest score, since the maxima are distinct scores of the row;
//   3. the scores >= tau (about 9 per group and half) are compacted into
//      per-lane shared-memory slots by predicated stores, the TMEM buffers
//      are released and the slots sorted by a network on packed keys.  A
//      warp where some row has more than CAND_CAP candidates (ties, or
//      scores far from i.i.d.) folds the half from TMEM by exact insertion.
// The two groups swap their sorted lists and both merge them; after both
// halves the top k of the candidate grid is taken by merge networks split
// between the groups, then the fp32 softmax and the ids.  A rows come from
// the query tensor map at h*a_stride_h + p*a_stride_p + t, column offset
// p*a_col_p; B rows from the key tensor map at p*K + key.
// With the split-bf16 layout A = [hi | lo] and each key box multiplies both
// halves, so S is the fp32 query . key product to ~2^-16.
constexpr int ROUTER_THREADS = 320;
// A stage holds ROUTER_KB K-columns of A (hi and, with the split layout, the
// matching lo columns) and of the keys; with the split layout one key box
// serves both the hi and the lo MMAs, so the keys cross L2 -> shared memory
// once.  The feed is bound by copy latency, not bandwidth, so the same 128 KB
// of ring is cut into more, narrower stages: 32 columns (64-byte rows, the
// 64-byte swizzle) x 4 stages keep 96 KB in flight where 64 x 2 kept 64 KB.
#ifndef ETHOS_ROUTER_KB
#define ETHOS_ROUTER_KB 32
#endif
constexpr int ROUTER_KB = ETHOS_ROUTER_KB;
static_assert(ROUTER_KB == 16 || ROUTER_KB == 32 || ROUTER_KB == 64, "stage width is one swizzle row");
constexpr int ROUTER_STAGES = 128 / ROUTER_KB;
constexpr int ROUTER_A_BYTES = 128 * ROUTER_KB * 2;
constexpr int ROUTER_B_BYTES_MAX = 256 * ROUTER_KB * 2;
constexpr int ROUTER_STAGE_BYTES = 2 * ROUTER_A_BYTES + ROUTER_B_BYTES_MAX;
// candidate slots per lane: CAND_CAP plus 4 of headroom (the count saturates
// once per 4 scores), (score, id) pairs laid out [slot][lane]; the fallback
// fold's 32 x 32 score staging aliases the same per-warp region
constexpr int CAND_CAP = 20;
constexpr int CAND_SLOTS = CAND_CAP + 4;
constexpr int ROUTER_CAND_WARP_BYTES = CAND_SLOTS * 32 * 8;
static_assert(ROUTER_CAND_WARP_BYTES >= 32 * 32 * 4, "fallback staging must fit the candidate region");
constexpr int ROUTER_CAND_BYTES = 8 * ROUTER_CAND_WARP_BYTES;
constexpr int ROUTER_XMAX_BYTES = 2 * 16 * 128 * 4;     // [group][16 maxima][128 rows]
constexpr int ROUTER_XLIST_BYTES = 2 * 16 * 128 * 4;    // [value|id][16][128 rows]

__device__ __forceinline__ uint64_t router_desc(uint32_t smem_addr) {
  return ROUTER_KB == 64 ? umma_desc_sw128(smem_addr)
                         : (ROUTER_KB == 32 ? umma_desc_sw64(smem_addr) : umma_desc_sw32(smem_addr));
}

struct RouterCtl {
  uint64_t full[ROUTER_STAGES];
  uint64_t empty[ROUTER_STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr int ROUTER_OFF_CAND = ROUTER_STAGES * ROUTER_STAGE_BYTES;
constexpr int ROUTER_OFF_XMAX = ROUTER_OFF_CAND + ROUTER_CAND_BYTES;
constexpr int ROUTER_OFF_XLIST = ROUTER_OFF_XMAX + ROUTER_XMAX_BYTES;
constexpr int ROUTER_OFF_CTL = ROUTER_OFF_XLIST + ROUTER_XLIST_BYTES;
constexpr int ROUTER_SMEM_BYTES = ROUTER_OFF_CTL + static_cast<int>(sizeof(RouterCtl)) + 1024;

struct RouterGeom {
  int T;          // tokens
  int H;          // heads
  int K;          // sub-keys per table
  int KA;         // contraction length of one score (dq for hi/lo, dq/2 plain)
  int a_stride_h; // A row offset per head
  int a_stride_p; // A row offset per half
  int a_col_p;    // A column offset per half
  int split;      // 1: A = [hi | lo] (KA columns), keys in columns [0, KA / 2)
};

template <int TOPK>
__global__ void __launch_bounds__(ROUTER_THREADS, 1)
    k_score_topk(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, RouterGeom g,
                 int32_t* __restrict__ ids_out, float* __restrict__ w_out, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  RouterCtl* ctl = reinterpret_cast<RouterCtl*>(smem + ROUTER_OFF_CTL);
  const int warp = warp_id();
  const int lane = lane_id();
  const int num_mt = (g.T + 127) / 128;
  const int num_items = g.H * num_mt;
  const int box_rows = g.K < 256 ? g.K : 256;   // keys per unit (TMA box rows, MMA N)
  const int num_chunks = (g.K + 255) / 256;     // units per half (1 or 2)
  const int num_kb = (g.split ? g.KA / 2 : g.KA) / ROUTER_KB;  // stages per unit
  const uint32_t stage_tx = (g.split ? 2 : 1) * ROUTER_A_BYTES + box_rows * ROUTER_KB * 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ROUTER_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], 256);  // all 8 epilogue warps consume every unit
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
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
      for (int item = blockIdx.x; ok && item < num_items; item += gridDim.x) {
        const int h = item / num_mt;
        const int t0 = (item - h * num_mt) * 128;
        for (int p = 0; ok && p < 2; ++p) {
          const int a_row = h * g.a_stride_h + p * g.a_stride_p + t0;
          for (int nc = 0; ok && nc < num_chunks; ++nc) {
            for (int kb = 0; kb < num_kb; ++kb) {
              if (!mbar_wait(&ctl->empty[rp.stage], rp.phase ^ 1u, abort, err, 11)) {
                ok = false;
                break;
              }
              uint8_t* sa = smem + rp.stage * ROUTER_STAGE_BYTES;
              mbar_arrive_expect_tx(&ctl->full[rp.stage], stage_tx);
              const int kc = kb * ROUTER_KB;
              tma_load_2d(sa, &tmA, &ctl->full[rp.stage], p * g.a_col_p + kc, a_row);
              if (g.split) tma_load_2d(sa + ROUTER_A_BYTES, &tmA, &ctl->full[rp.stage], g.KA / 2 + kc, a_row);
              tma_load_2d(sa + 2 * ROUTER_A_BYTES, &tmB, &ctl->full[rp.stage], kc, p * g.K + nc * 256);
              rp.advance(ROUTER_STAGES);
            }
          }
        }
      }
      if (!ok) rp.drain(ctl->full, ROUTER_STAGES, err, 15);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(128, box_rows);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < num_items; item += gridDim.x) {
        for (int u = 0; ok && u < 2 * num_chunks; ++u, ++it) {
          const int buf = it & 1;
          const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
          if (!mbar_wait(&ctl->acc_empty[buf], acc_phase ^ 1u, abort, err, 12)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * 256);
          for (int kb = 0; kb < num_kb; ++kb) {
            if (!mbar_wait(&ctl->full[stage], phase, abort, err, 13)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(smem + stage * ROUTER_STAGE_BYTES);
            const uint32_t b_base = a_base + 2 * ROUTER_A_BYTES;
#pragma unroll
            for (int k = 0; k < ROUTER_KB / 16; ++k) {
              umma_bf16(d, router_desc(a_base + k * 32), router_desc(b_base + k * 32), idesc,
                        (kb | k) != 0 ? 1u : 0u);
            }
            if (g.split) {
#pragma unroll
              for (int k = 0; k < ROUTER_KB / 16; ++k)
                umma_bf16(d, router_desc(a_base + ROUTER_A_BYTES + k * 32), router_desc(b_base + k * 32), idesc, 1u);
            }
            umma_commit(&ctl->empty[stage]);
            if (++stage == ROUTER_STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&ctl->acc_full[buf]);
        }
      }
      if (!ok || *abort) {
        umma_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr, err, 16);
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    // Both groups work on every unit: group grp takes columns [128 grp,
    // 128 grp + 128) of it.  All their exchanges go through shared memory
    // between two syncs of named barrier 1 (256 threads): the first makes
    // sure the previous readers of the region are done, the second publishes
    // the writes.  Every warp walks all items and takes every sync in the
    // same order, also after an abort (work is skipped, syncs are not).
    const int ew = warp - 2;
    const int q = warp & 3;    // TMEM lane quarter = rows of this warp
    const int grp = ew >> 2;   // column half of every unit
    const int row = q * 32 + lane;
    uint8_t* wreg = smem + ROUTER_OFF_CAND + ew * ROUTER_CAND_WARP_BYTES;
    float2* cand = reinterpret_cast<float2*>(wreg) + lane;  // slot s at cand[32 * s]
    float* stage = reinterpret_cast<float*>(wreg);           // fallback staging [32][32]
    float* xmax = reinterpret_cast<float*>(smem + ROUTER_OFF_XMAX);   // [2][16][128] maxima
    // 16 (score, id) pairs per row: group 0 publishes through the list
    // region, group 1 through the maxima region (free at that point)
    float* pub_v = reinterpret_cast<float*>(smem + (grp == 0 ? ROUTER_OFF_XLIST : ROUTER_OFF_XMAX));
    int* pub_i = reinterpret_cast<int*>(pub_v) + 16 * 128;
    const float* oth_v = reinterpret_cast<const float*>(smem + (grp == 0 ? ROUTER_OFF_XMAX : ROUTER_OFF_XLIST));
    const int* oth_i = reinterpret_cast<const int*>(oth_v) + 16 * 128;
    int m = 0;   // units consumed
    int it = 0;  // items walked
    bool ok = true;
    for (int item = blockIdx.x; item < num_items; item += gridDim.x, ++it) {
      const int h = item / num_mt;
      const int t = (item - h * num_mt) * 128 + row;
      // The half loop stays rolled (one copy of its body in the instruction
      // stream): the current half's list is (cv, ci), half 0's is copied to
      // (lv0, li0) at the end of its iteration and half 1's stays in (cv, ci).
      float lv0[TOPK], cv[TOPK];
      int li0[TOPK], ci[TOPK];
#pragma unroll 1
      for (int p = 0; p < 2; ++p) {
#pragma unroll
        for (int j = 0; j < TOPK; ++j) {
          cv[j] = -INFINITY;
          ci[j] = 0;
        }
        // The half's units stay in TMEM until its candidates are compacted:
        // 1. per unit, the maxima of this group's 8-key groups, sorted and
        //    merged into the top 16 over the half's units;
        // 2. tau = TOPK-th largest of the half's 8-key maxima (both groups,
        //    exchanged): a lower bound on the half's TOPK-th largest score,
        //    since the maxima are distinct scores of the row, so every score
        //    of the half's top TOPK is >= tau (about 9 of this group's 256
        //    scores pass);
        // 3. the scores >= tau of all the half's units are compacted into
        //    this lane's shared-memory slots, the buffers are released and
        //    the slots are sorted into this group's list for the half.
        const int m0 = m;
        m += num_chunks;
        float t16[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) t16[i] = -INFINITY;
        for (int nc = 0; nc < num_chunks; ++nc) {
          const int buf = (m0 + nc) & 1;
          const uint32_t ph = static_cast<uint32_t>((m0 + nc) >> 1) & 1u;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&ctl->acc_full[buf], ph, abort, err, 14));
          if (ok) tc_fence_after();
          const int valid = min(256, g.K - nc * 256);                // multiple of 32
          const int vg = min(128, max(0, valid - 128 * grp));        // this group's columns
          const uint32_t cbase = tmem_addr(tmem, q * 32, buf * 256 + 128 * grp);
          float mx[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) mx[i] = -INFINITY;
          if (ok) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              if (c * 64 < vg) {  // a 32-column tail reads 32 spare columns
                float sc[64];
                tmem_ld64(cbase + c * 64, sc);
#pragma unroll
                for (int g8 = 0; g8 < 8; ++g8) {
                  const float* v = sc + 8 * g8;
                  const float mv = fmax3(fmax3(v[0], v[1], v[2]), fmax3(v[3], v[4], v[5]), fmaxf(v[6], v[7]));
                  mx[8 * c + g8] = (c * 64 + 8 * g8 < vg) ? mv : -INFINITY;
                }
              }
            }
          }
          bitonic_sort_desc<16>(mx);
          if (nc == 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) t16[i] = mx[i];
          } else {
            // top 16 of two sorted lists: max(a_i, b_15-i) is bitonic, then
            // the half-cleaner merge
#pragma unroll
            for (int i = 0; i < 16; ++i) t16[i] = fmaxf(t16[i], mx[15 - i]);
#pragma unroll
            for (int j = 8; j > 0; j >>= 1) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if ((i & j) == 0) {
                  const float x = t16[i], y = t16[i | j];
                  t16[i] = fmaxf(x, y);
                  t16[i | j] = fminf(x, y);
                }
              }
            }
          }
        }
        named_bar_sync(1, 256);
#pragma unroll
        for (int i = 0; i < 16; ++i) xmax[(grp * 16 + i) * 128 + row] = t16[i];
        named_bar_sync(1, 256);
        float tau = -INFINITY;
        if (g.K / 8 >= TOPK) {
          tau = INFINITY;
#pragma unroll
          for (int i = 0; i < TOPK; ++i)
            tau = fminf(tau, fmaxf(t16[i], xmax[((grp ^ 1) * 16 + TOPK - 1 - i) * 128 + row]));
        }
        if (ok) {
          // Predicated and branch-free: a passing score is stored with its
          // key id into the next free slot (8-byte slots, [slot][lane] rows
          // of 256 B) and the slot address advances; rejected scores issue
          // no shared-memory traffic.  The address saturates at CAND_CAP
          // once per 4 scores (CAND_SLOTS covers the 4 in between); a
          // saturated row is an overflow.
          const uint32_t c0 = smem_u32(cand);
          const uint32_t ccap = c0 + CAND_CAP * 256u;
          uint32_t ca = c0;
          int fold_from = num_chunks;  // first unit that overflowed (num_chunks: none)
#pragma unroll 1
          for (int nc = 0; nc < num_chunks; ++nc) {
            const int buf = (m0 + nc) & 1;
            const int valid = min(256, g.K - nc * 256);
            const int vg = min(128, max(0, valid - 128 * grp));
            const int key0 = nc * 256 + 128 * grp;
            const uint32_t cbase = tmem_addr(tmem, q * 32, buf * 256 + 128 * grp);
            const uint32_t ca_unit = ca;
            bool over = false;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              if (c * 64 >= vg) break;
              float sc[64];
              tmem_ld64(cbase + c * 64, sc);
              int id = key0 + c * 64;
              const int ng = min(16, (vg - c * 64) / 4);
#pragma unroll
              for (int g4 = 0; g4 < 16; ++g4) {
                if (g4 >= ng) break;
#pragma unroll
                for (int i = 0; i < 4; ++i, ++id) {
                  asm volatile(
                      "{\n\t.reg .pred p;\n\t"
                      "setp.ge.f32 p, %1, %2;\n\t"
                      "@p st.shared.v2.b32 [%0], {%1, %3};\n\t"
                      "@p add.u32 %0, %0, 256;\n\t}"
                      : "+r"(ca)
                      : "f"(sc[4 * g4 + i]), "f"(tau), "r"(id)
                      : "memory");
                }
                over |= ca > ccap;
                ca = ca > ccap ? ccap : ca;
              }
            }
            if (__any_sync(0xffffffffu, over)) {
              ca = ca_unit;  // this unit and the later ones are folded from TMEM
              fold_from = nc;
              break;
            }
            tc_fence_before();
            mbar_arrive(&ctl->acc_empty[buf]);  // the unit's scores are no longer needed
          }
          const int n = static_cast<int>((ca - c0) >> 8);
          if (fold_from == num_chunks) {
            // Sort keys, not (score, id) pairs: each candidate's slot number
            // rides in the 5 low mantissa bits of its score, so a min/max
            // network (2 instructions per exchange instead of 5) orders them,
            // and the exact score and id are fetched back by slot.  A key
            // differs from its score by < 32 ulps, which can only reorder
            // candidates that close; unused slots get finite -FLT_MAX keys
            // carrying their own slot (>= n), never NaN.
            static_assert(CAND_CAP <= 32, "slot numbers use 5 key bits");
            float key[16];
#pragma unroll
            for (int s2 = 0; s2 < 16; ++s2) {
              const float sc = s2 < n ? cand[32 * s2].x : -FLT_MAX;
              key[s2] = __uint_as_float((__float_as_uint(sc) & ~31u) | static_cast<uint32_t>(s2));
            }
            bitonic_sort_desc<16>(key);
            if (__any_sync(0xffffffffu, n > 16)) {  // slots 16..19 in use somewhere in the warp
              float k4[16];
#pragma unroll
              for (int s2 = 0; s2 < 16; ++s2) k4[s2] = -FLT_MAX;
#pragma unroll
              for (int s2 = 0; s2 < CAND_CAP - 16; ++s2) {
                const float sc = 16 + s2 < n ? cand[32 * (16 + s2)].x : -FLT_MAX;
                k4[s2] = __uint_as_float((__float_as_uint(sc) & ~31u) | static_cast<uint32_t>(16 + s2));
              }
              {
                float t4[4];
#pragma unroll
                for (int s2 = 0; s2 < 4; ++s2) t4[s2] = k4[s2];
                bitonic_sort_desc<4>(t4);
#pragma unroll
                for (int s2 = 0; s2 < 4; ++s2) k4[s2] = t4[s2];
              }
              // top 16 of the two sorted key lists (max(a_i, b_15-i) is
              // bitonic), then the half-cleaner merge
#pragma unroll
              for (int i = 0; i < 16; ++i) key[i] = fmaxf(key[i], k4[15 - i]);
#pragma unroll
              for (int j = 8; j > 0; j >>= 1) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  if ((i & j) == 0) {
                    const float x = key[i], y = key[i | j];
                    key[i] = fmaxf(x, y);
                    key[i | j] = fminf(x, y);
                  }
                }
              }
            }
#pragma unroll
            for (int j = 0; j < TOPK; ++j) {
              const int slot = static_cast<int>(__float_as_uint(key[j]) & 31u);
              const float2 e = cand[32 * slot];
              cv[j] = slot < n ? e.x : -INFINITY;
              ci[j] = slot < n ? __float_as_int(e.y) : 0;
            }
          } else {
            // Rare: some row of the warp has more than CAND_CAP candidates.
            // The candidates of the units already compacted are inserted
            // from their slots, the rest of the half is folded from TMEM by
            // exact insertion, and those units are released.
            __syncwarp();
            const int nmax = __reduce_max_sync(0xffffffffu, n);
#pragma unroll 1
            for (int s2 = 0; s2 < nmax; ++s2) {
              const float2 e = cand[32 * s2];
              topk_insert<TOPK>(cv, ci, s2 < n ? e.x : -INFINITY, s2 < n ? __float_as_int(e.y) : 0);
            }
            __syncwarp();
#pragma unroll 1
            for (int nc = fold_from; nc < num_chunks; ++nc) {
              const int buf = (m0 + nc) & 1;
              const int valid = min(256, g.K - nc * 256);
              const int vg = min(128, max(0, valid - 128 * grp));
              const int key0 = nc * 256 + 128 * grp;
              const uint32_t cbase = tmem_addr(tmem, q * 32, buf * 256 + 128 * grp);
#pragma unroll 1
              for (int c = 0; c < 4; ++c) {
                if (c * 32 >= vg) break;
                float sc[32];
                tmem_ld32(cbase + c * 32, sc);
                topk_fold_chunk<TOPK, false>(cv, ci, sc, nullptr, key0 + c * 32, tau, stage, nullptr, lane);
              }
              tc_fence_before();
              mbar_arrive(&ctl->acc_empty[buf]);
            }
          }
          __syncwarp();
        }
        // 4. the two groups swap their half-p lists and both merge them,
        //    both with group 0's list as the first operand: with tied scores
        //    the merge order decides which of the tied entries lands where,
        //    and the split grid step needs the same list in both groups
        named_bar_sync(1, 256);
#pragma unroll
        for (int j = 0; j < TOPK; ++j) {
          pub_v[j * 128 + row] = cv[j];
          pub_i[j * 128 + row] = ci[j];
        }
        named_bar_sync(1, 256);
        {
          float ov[TOPK];
          int oi[TOPK];
#pragma unroll
          for (int j = 0; j < TOPK; ++j) {
            ov[j] = oth_v[j * 128 + row];
            oi[j] = oth_i[j * 128 + row];
          }
          if (grp == 0) {
            top_merge_kv<TOPK>(cv, ci, ov, oi);
          } else {
            top_merge_kv<TOPK>(ov, oi, cv, ci);
#pragma unroll
            for (int j = 0; j < TOPK; ++j) {
              cv[j] = ov[j];
              ci[j] = oi[j];
            }
          }
        }
        if (p == 0) {
#pragma unroll
          for (int j = 0; j < TOPK; ++j) {
            lv0[j] = cv[j];
            li0[j] = ci[j];
          }
        }
      }
      // 5. top TOPK of the candidate grid; for TOPK = 16 the merge tree is
      //    split: the helper group merges rows 2..7 and publishes them, the
      //    finishing group (alternating per item) merges rows 0, 1 and the
      //    singles, then the helper's list, and writes the result
      const int fin = it & 1;
      float fv[TOPK];
      int fid[TOPK];
      if constexpr (TOPK == 16) {
        if (grp == fin) {
          grid_rows01<16>(lv0, li0, cv, ci, g.K, fv, fid);
        } else {
          grid_rows27<16>(lv0, li0, cv, ci, g.K, fv, fid);
        }
        named_bar_sync(1, 256);
        if (grp != fin) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            pub_v[j * 128 + row] = fv[j];
            pub_i[j * 128 + row] = fid[j];
          }
        }
        named_bar_sync(1, 256);
        if (grp == fin) {
          float ov[16];
          int oi[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            ov[j] = oth_v[j * 128 + row];
            oi[j] = oth_i[j * 128 + row];
          }
          top_merge_kv<16>(fv, fid, ov, oi);
        }
      } else {
        if (grp == fin) grid_topk<TOPK>(lv0, li0, cv, ci, g.K, fv, fid);
      }
      if (grp == fin && ok && t < g.T) {
        // fp32 softmax over the selected scores (model.py:234)
        float e[TOPK];
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < TOPK; ++j) {
          e[j] = expf(fv[j] - fv[0]);
          sum += e[j];
        }
        const float inv = __frcp_rn(sum);  // e / sum to within an ulp
        const int64_t o = (static_cast<int64_t>(t) * g.H + h) * TOPK;
        int4* di = reinterpret_cast<int4*>(ids_out + o);
        float4* dw = reinterpret_cast<float4*>(w_out + o);
#pragma unroll
        for (int j = 0; j < TOPK / 4; ++j) {
          di[j] = make_int4(fid[4 * j], fid[4 * j + 1], fid[4 * j + 2], fid[4 * j + 3]);
          dw[j] = make_float4(e[4 * j] * inv, e[4 * j + 1] * inv, e[4 * j + 2] * inv, e[4 * j + 3] * inv);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------- BatchNorm (training) --
// Column statistics of qpre [T, C] (C = H*dq) in two passes over row slabs.
// Pass 1: per (slab, column) shifted sums around the column's first value
// (a cheap pivot that keeps the one-pass variance well conditioned).
// Partial sums land in part[slab][C][2]; k_bn_finalize combines them.
constexpr int BN_ROWS_PER_SLAB = 256;

__global__ void k_bn_partial(const float* __restrict__ qpre, int T, int C, float* __restrict__ part) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int slab = blockIdx.y;
  if (col >= C) return;
  const float pivot = qpre[col];
  const int r0 = slab * BN_ROWS_PER_SLAB;
  const int r1 = min(T, r0 + BN_ROWS_PER_SLAB);
  float s = 0.f, ss = 0.f;
  for (int r = r0; r < r1; ++r) {
    const float d = qpre[static_cast<int64_t>(r) * C + col] - pivot;
    s += d;
    ss = fmaf(d, d, ss);
  }
  part[(static_cast<int64_t>(slab) * C + col) * 2 + 0] = s;
  part[(static_cast<int64_t>(slab) * C + col) * 2 + 1] = ss;
}

// Combines the slab sums (in double), writes the batch mean and 1/sqrt(var +
// eps) (biased variance, as BatchNorm1d normalises), the fused per-column
// (scale, offset) of the normalisation pass, and updates the running
// statistics with the unbiased variance.
__global__ void k_bn_finalize(const float* __restrict__ qpre, const float* __restrict__ part, int T, int C,
                              int slabs, const float* __restrict__ gamma, const float* __restrict__ beta,
                              float* __restrict__ run_mean, float* __restrict__ run_var, float eps,
                              float momentum, float* __restrict__ save_bn, float2* __restrict__ colp) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= C) return;
  double s = 0.0, ss = 0.0;
  for (int k = 0; k < slabs; ++k) {
    s += part[(static_cast<int64_t>(k) * C + col) * 2 + 0];
    ss += part[(static_cast<int64_t>(k) * C + col) * 2 + 1];
  }
  const double pivot = qpre[col];
  const double md = s / T;
  double var = ss / T - md * md;
  if (var < 0.0) var = 0.0;
  const float mean = static_cast<float>(pivot + md);
  const float invstd = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
  save_bn[col] = mean;
  save_bn[C + col] = invstd;
  const float scale = invstd * gamma[col];
  colp[col] = make_float2(scale, beta[col] - mean * scale);
  const double unbiased = T > 1 ? var * T / (T - 1) : var;
  run_mean[col] = (1.f - momentum) * run_mean[col] + momentum * mean;
  run_var[col] = (1.f - momentum) * run_var[col] + momentum * static_cast<float>(unbiased);
}

// Eval-mode per-column (scale, offset) from the bias and running statistics:
// ((v + bias) - rm) * gamma / sqrt(rv + eps) + beta = v * scale + offset.
// With on_qpre != 0 the affine applies to qpre = v + bias instead.
__global__ void k_bn_eval_colp(const float* __restrict__ bn, int C, float eps, int on_qpre,
                               float2* __restrict__ colp) {
  pdl_launch_dependents();
  pdl_wait();
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= C) return;
  const float bias = on_qpre ? 0.f : bn[col], gamma = bn[1 * C + col], beta = bn[2 * C + col];
  const float rm = bn[3 * C + col], rv = bn[4 * C + col];
  const float scale = gamma / sqrtf(rv + eps);
  colp[col] = make_float2(scale, beta - (rm - bias) * scale);
}

// Training-mode (scale, offset) from the batch statistics a forward saved
// (mean, 1/sqrt(var + eps)), computed exactly as k_bn_finalize computes them,
// so that a backward recomputing q^ from qpre gets the forward's values.
__global__ void k_bn_colp_from_stats(const float* __restrict__ bn, const float* __restrict__ stats, int C,
                                     float2* __restrict__ colp) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= C) return;
  const float scale = stats[C + col] * bn[C + col];
  colp[col] = make_float2(scale, bn[2 * C + col] - stats[col] * scale);
}

// Normalisation pass on qpre [T, C] -> split-bf16 scoring operand
// qs[p][h][t][hi | lo].  One thread per 8 consecutive columns.
// Grid: x covers the column groups of 8 (blockDim.x threads each), y walks the
// token rows, so the per-thread column math (head, half, offset) is computed
// once and no thread divides by runtime sizes inside the row loop.
__global__ void k_bn_apply(const float* __restrict__ qpre, const float2* __restrict__ colp, int T, int H, int dq,
                           __nv_bfloat16* __restrict__ qs) {
  const int C = H * dq;
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= C) return;
  const int h = col / dq;
  const int e = col - h * dq;
  const int half = dq >> 1;
  const int p = e >= half ? 1 : 0;
  const int i0 = e - p * half;
  float2 cp[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) cp[u] = colp[col + u];
  __nv_bfloat16* qbase = qs + static_cast<int64_t>(p * H + h) * T * dq;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const float4* src = reinterpret_cast<const float4*>(qpre + static_cast<int64_t>(t) * C + col);
    const float4 a = src[0], b = src[1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const float q0 = fmaf(v[i], cp[i].x, cp[i].y);
      const float q1 = fmaf(v[i + 1], cp[i + 1].x, cp[i + 1].y);
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(q0, q1);
      const float2 hf = __bfloat1622float2(h2);
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(q0 - hf.x, q1 - hf.y);
      hi[i >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
      lo[i >> 1] = *reinterpret_cast<const uint32_t*>(&l2);
    }
    __nv_bfloat16* base = qbase + static_cast<int64_t>(t) * dq;
    *reinterpret_cast<uint4*>(base + i0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(base + half + i0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

}  // namespace ethos
