// Product-key router kernels: sub-key scoring on tcgen05 with a fused top-k
// epilogue (per-half top-k, candidate-grid top-k, fp32 softmax, id decode),
// and the BatchNorm batch-statistics / normalisation kernels of training mode.
//
// Reference: ProductKeyRouter.forward, model.py:208-254.
#pragma once

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

// N-th largest of the 2N values a[0..N) and b[0..N) (N a power of two): sort
// both descending with a bitonic network, then the N-th largest of the union
// is min_i max(a[i], b[N-1-i]).
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
template <int N>
__device__ __forceinline__ float nth_largest_of_union(float (&a)[N], float (&b)[N]) {
  bitonic_sort_desc<N>(a);
  bitonic_sort_desc<N>(b);
  float t = INFINITY;
#pragma unroll
  for (int i = 0; i < N; ++i) t = fminf(t, fmaxf(a[i], b[N - 1 - i]));
  return t;
}

// ------------------------------------------------------ scoring + top-k --
// One work item = (head h, tile of 128 tokens); per item two halves p, per
// half the sub-keys in units of up to 256 (TMEM buffer = unit parity).
// The MMA warp computes S[t, key] = sum_c A[t, c] * B[key, c] into the
// unit's 256-column TMEM buffer; 8 epilogue warps (one token row per thread,
// group kh = 0/1 owning the first/second 256 keys of a half) select the
// half's top-k per row exactly in three steps:
//   1. maxima of the 16-key groups of the row (one FMNMX per score);
//   2. tau = k-th largest of those 32 maxima (a lower bound on the k-th
//      largest score, since the maxima are k+ distinct scores of the row);
//   3. fold only scores >= tau into a sorted register list (the threshold
//      leaves ~20 candidates per 512 keys instead of ~150).
// Group 1 then hands its list to group 0, which merges the two, and after
// both halves forms the candidate grid, the fp32 softmax and the ids.  A
// rows come from the query tensor map at h*a_stride_h + p*a_stride_p + t,
// column offset p*a_col_p; B rows from the key tensor map at p*K + key.
// With the split-bf16 layout A = [hi | lo] and B = [keys | keys], so S is the
// fp32 query . key product to ~2^-16.
constexpr int ROUTER_THREADS = 320;
constexpr int ROUTER_STAGES = 3;
constexpr int ROUTER_A_BYTES = 128 * 64 * 2;
constexpr int ROUTER_B_BYTES_MAX = 256 * 64 * 2;
constexpr int ROUTER_STAGE_BYTES = ROUTER_A_BYTES + ROUTER_B_BYTES_MAX;
// candidate staging: 32 x 32 fp32 scores per epilogue warp, plus 32 x 32 int
// ids for the 4 warps of group 0 (merges and the candidate grid)
constexpr int ROUTER_CAND_BYTES = 8 * 32 * 32 * 4 + 4 * 32 * 32 * 4;
constexpr int ROUTER_XMAX_BYTES = 2 * 16 * 128 * 4;     // [group][16 maxima][128 rows]
constexpr int ROUTER_XLIST_BYTES = 2 * 16 * 128 * 4;    // [value|id][16][128 rows]

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
};

__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

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
  const int num_kb = g.KA / 64;
  const uint32_t stage_tx = ROUTER_A_BYTES + box_rows * 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ROUTER_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], 128);  // one warp group (4 warps) consumes a unit
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
              tma_load_2d(sa, &tmA, &ctl->full[rp.stage], p * g.a_col_p + kb * 64, a_row);
              tma_load_2d(sa + ROUTER_A_BYTES, &tmB, &ctl->full[rp.stage], kb * 64, p * g.K + nc * 256);
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
            const uint32_t b_base = a_base + ROUTER_A_BYTES;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              umma_bf16(d, umma_desc_sw128(a_base + k * 32), umma_desc_sw128(b_base + k * 32), idesc,
                        (kb | k) != 0 ? 1u : 0u);
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
    // Every participating warp walks all items and hits every named barrier,
    // also after an abort (work is skipped, barriers are not).
    const int ew = warp - 2;
    const int q = warp & 3;
    const int kh = ew >> 2;  // key group: units with nc == kh
    const bool two = num_chunks == 2;
    if (!two && kh == 1) {
      // one unit per half: group 0 alone handles every unit
    } else {
      const int row = q * 32 + lane;
      float* stage = reinterpret_cast<float*>(smem + ROUTER_OFF_CAND) + ew * 32 * 32;
      int* stage_id = reinterpret_cast<int*>(smem + ROUTER_OFF_CAND + 8 * 32 * 32 * 4) + (ew & 3) * 32 * 32;
      float* xmax = reinterpret_cast<float*>(smem + ROUTER_OFF_XMAX);   // [2][16][128]
      float* xlv = reinterpret_cast<float*>(smem + ROUTER_OFF_XLIST);   // [16][128]
      int* xli = reinterpret_cast<int*>(smem + ROUTER_OFF_XLIST) + 16 * 128;
      int m = 0;  // units consumed by this group
      bool ok = true;
      for (int item = blockIdx.x; item < num_items; item += gridDim.x) {
        const int h = item / num_mt;
        const int t = (item - h * num_mt) * 128 + row;
        float lv[2][TOPK];
        int li[2][TOPK];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
#pragma unroll
          for (int j = 0; j < TOPK; ++j) {
            lv[p][j] = -INFINITY;
            li[p][j] = 0;
          }
          for (int nc = (two ? kh : 0); nc < num_chunks; nc += (two ? 2 : 1), ++m) {
            // unit index within this CTA's sequence: two groups alternate
            // buffers 0/1 (two == true) or one group walks both buffers
            const int buf = two ? kh : (m & 1);
            const uint32_t ph = two ? (static_cast<uint32_t>(m) & 1u) : (static_cast<uint32_t>(m >> 1) & 1u);
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&ctl->acc_full[buf], ph, abort, err, 14));
            const int valid = min(256, g.K - nc * 256);
            const int key_base = nc * 256;
            const uint32_t cbase = tmem_addr(tmem, q * 32, buf * 256);
            if (ok) tc_fence_after();
            // 1. maxima of 16-key groups
            float mx[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) mx[i] = -INFINITY;
            if (ok) {
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                if (c * 32 < valid) {
                  float sc[32];
                  tmem_ld32(cbase + c * 32, sc);
                  float m0 = sc[0], m1 = sc[16];
#pragma unroll
                  for (int i = 1; i < 16; ++i) {
                    m0 = fmaxf(m0, sc[i]);
                    m1 = fmaxf(m1, sc[16 + i]);
                  }
                  mx[2 * c] = m0;
                  mx[2 * c + 1] = m1;
                }
              }
            }
            // 2. tau = TOPK-th largest of the row's 16-key maxima (both groups)
            float tau;
            if (two) {
#pragma unroll
              for (int i = 0; i < 16; ++i) xmax[(kh * 16 + i) * 128 + row] = mx[i];
              named_bar_sync(1, 256);
              float other[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) other[i] = xmax[((kh ^ 1) * 16 + i) * 128 + row];
              if (TOPK == 16) {
                tau = nth_largest_of_union<16>(mx, other);
              } else {
                bitonic_sort_desc<16>(mx);
                bitonic_sort_desc<16>(other);
                float u[2 * TOPK];  // TOPK-th largest of the merged top lists
#pragma unroll
                for (int i = 0; i < TOPK; ++i) {
                  u[i] = mx[i];
                  u[TOPK + i] = other[i];
                }
                float a_[TOPK], b_[TOPK];
#pragma unroll
                for (int i = 0; i < TOPK; ++i) {
                  a_[i] = u[i];
                  b_[i] = u[TOPK + i];
                }
                tau = nth_largest_of_union<TOPK>(a_, b_);
              }
            } else {
              // one unit per half: maxima of this unit only (valid/16 of them)
              const int nmax = valid / 16;
              if (nmax >= TOPK) {
                bitonic_sort_desc<16>(mx);
                tau = mx[TOPK - 1];
              } else {
                tau = -INFINITY;
              }
            }
            // 3. fold scores >= tau
            if (ok) {
#pragma unroll 1
              for (int c = 0; c < 8; ++c) {
                if (c * 32 >= valid) break;
                float sc[32];
                tmem_ld32(cbase + c * 32, sc);
                topk_fold_chunk<TOPK, false>(lv[p], li[p], sc, nullptr, key_base + c * 32, tau, stage, stage_id,
                                             lane);
              }
              tc_fence_before();
              mbar_arrive(&ctl->acc_empty[buf]);
            }
          }
          if (two) {
            // group 1 hands its half-p list to group 0
            if (kh == 1) {
#pragma unroll
              for (int j = 0; j < TOPK; ++j) {
                xlv[j * 128 + row] = lv[p][j];
                xli[j * 128 + row] = li[p][j];
              }
              named_bar_sync(2, 256);
            } else {
              named_bar_sync(2, 256);
              float ov[32];
              int oi[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                ov[j] = j < TOPK ? xlv[j * 128 + row] : -INFINITY;
                oi[j] = j < TOPK ? xli[j * 128 + row] : 0;
              }
              topk_fold_chunk<TOPK, true>(lv[p], li[p], ov, oi, 0, -INFINITY, stage, stage_id, lane);
            }
          }
        }
        if (kh == 0) {
          // Top-k of the candidate grid lv[0][i] + lv[1][j].  Only pairs with
          // (i+1)(j+1) <= TOPK can rank in the top TOPK (every (i', j') with
          // i' <= i, j' <= j scores at least as high); tau_c = max(a_0 +
          // b_{k-1}, a_{k-1} + b_0) bounds the k-th largest sum from below.
          constexpr int NC = (TOPK == 16) ? 50 : (TOPK == 8 ? 20 : 8);
          float cv[64];
          int ci[64];
          int n = 0;
#pragma unroll
          for (int i = 0; i < TOPK; ++i) {
#pragma unroll
            for (int j = 0; (i + 1) * (j + 1) <= TOPK; ++j) {
              cv[n] = lv[0][i] + lv[1][j];
              ci[n] = li[0][i] * g.K + li[1][j];
              ++n;
            }
          }
#pragma unroll
          for (int j = NC; j < 64; ++j) {
            cv[j] = -INFINITY;
            ci[j] = 0;
          }
          const float tau_c = fmaxf(lv[0][0] + lv[1][TOPK - 1], lv[0][TOPK - 1] + lv[1][0]);
          float fv[TOPK];
          int fid[TOPK];
#pragma unroll
          for (int j = 0; j < TOPK; ++j) {
            fv[j] = -INFINITY;
            fid[j] = 0;
          }
          {
            float c0[32], c1[32];
            int d0[32], d1[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              c0[j] = cv[j];
              d0[j] = ci[j];
              c1[j] = cv[32 + j];
              d1[j] = ci[32 + j];
            }
            topk_fold_chunk<TOPK, true>(fv, fid, c0, d0, 0, tau_c, stage, stage_id, lane);
            topk_fold_chunk<TOPK, true>(fv, fid, c1, d1, 0, tau_c, stage, stage_id, lane);
          }
          if (ok && t < g.T) {
            // fp32 softmax over the selected scores (model.py:234)
            float e[TOPK];
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < TOPK; ++j) {
              e[j] = expf(fv[j] - fv[0]);
              sum += e[j];
            }
            const int64_t o = (static_cast<int64_t>(t) * g.H + h) * TOPK;
            int4* di = reinterpret_cast<int4*>(ids_out + o);
            float4* dw = reinterpret_cast<float4*>(w_out + o);
#pragma unroll
            for (int j = 0; j < TOPK / 4; ++j) {
              di[j] = make_int4(fid[4 * j], fid[4 * j + 1], fid[4 * j + 2], fid[4 * j + 3]);
              dw[j] = make_float4(e[4 * j] / sum, e[4 * j + 1] / sum, e[4 * j + 2] / sum, e[4 * j + 3] / sum);
            }
          }
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
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= C) return;
  const float bias = on_qpre ? 0.f : bn[col], gamma = bn[1 * C + col], beta = bn[2 * C + col];
  const float rm = bn[3 * C + col], rv = bn[4 * C + col];
  const float scale = gamma / sqrtf(rv + eps);
  colp[col] = make_float2(scale, beta - (rm - bias) * scale);
}

// Normalisation pass on qpre [T, C] -> split-bf16 scoring operand
// qs[p][h][t][hi | lo].  One thread per 8 consecutive columns.
__global__ void k_bn_apply(const float* __restrict__ qpre, const float2* __restrict__ colp, int T, int H, int dq,
                           __nv_bfloat16* __restrict__ qs) {
  const int C = H * dq;
  const int groups = C / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(T) * groups) return;
  const int t = static_cast<int>(idx / groups);
  const int col = static_cast<int>(idx - static_cast<int64_t>(t) * groups) * 8;
  const int h = col / dq;
  const int e = col - h * dq;
  const int half = dq >> 1;
  const int p = e >= half ? 1 : 0;
  const int i0 = e - p * half;
  const float4* src = reinterpret_cast<const float4*>(qpre + static_cast<int64_t>(t) * C + col);
  const float4 a = src[0], b = src[1];
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    float qn[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float2 cp = colp[col + i + u];
      qn[u] = fmaf(v[i + u], cp.x, cp.y);
    }
    const __nv_bfloat162 h2 = __floats2bfloat162_rn(qn[0], qn[1]);
    const float2 hf = __bfloat1622float2(h2);
    const __nv_bfloat162 l2 = __floats2bfloat162_rn(qn[0] - hf.x, qn[1] - hf.y);
    hi[i >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
    lo[i >> 1] = *reinterpret_cast<const uint32_t*>(&l2);
  }
  __nv_bfloat16* base = qs + (static_cast<int64_t>(p * H + h) * T + t) * dq;
  *reinterpret_cast<uint4*>(base + i0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(base + half + i0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

}  // namespace ethos
