// Reordered hypernetwork-expert forward on tcgen05.
//
// Per token t (reference: SimplifiedHypernetMoE.forward, model.py:306-341;
// reordered form of paper Algorithm 1 / kernels.py:80-120):
//   z_r   = E[id_r]                         r = 0..R-1 (R = H*k selections)
//   pre_r = z_r @ W1^T                      [dh]   (W1 = net.0.weight [dh, dl])
//   h_r   = gelu_erf(pre_r)                        (model.py:323)
//   dot_r = h_r . xp_t                             (xp = x @ W_u, model.py:326)
//   a_r   = gelu_erf(dot_r) * w_r                  (model.py:329)
//   hacc_t = sum_r a_r h_r                  [dh]   (fed to y = hacc @ W_v / H)
//
// One persistent CTA per SM walks tokens blockIdx.x, +gridDim.x, ...  The
// token's R latent rows are gathered with 16-byte cp.async into a 128-row A
// tile (128-byte swizzle, zero rows past R); W1 stays resident in shared
// memory (128 KB); two M=128 x N=256 x K=128 MMAs put pre for all 512 hidden
// units of the token in TMEM (128 lanes x 512 columns).  Eight epilogue warps
// then (pass 1) apply GELU in place in TMEM and form the dot products, and
// (pass 2) reduce a_r * h_r over the 128 rows with warp transpose-reductions.
//
// Warp roles (384 threads): 0-1 gather producers, 2 TMEM owner + W1 loader +
// MMA issuer, 3 idle, 4-11 epilogue (warp w reads TMEM lanes 32*(w%4)..+31 and
// column group (w-4)/4).
#pragma once

#include "gemm.cuh"

namespace ethos {

constexpr int EX_DL = 128;
constexpr int EX_DH = 512;
constexpr int EX_ROWS = 128;
constexpr int EX_THREADS = 384;
constexpr int EX_W1_BYTES = EX_DH * EX_DL * 2;   // 131072
constexpr int EX_Z_BYTES = EX_ROWS * EX_DL * 2;  // 32768
constexpr int EX_ZSTAGES = 2;
constexpr int EX_OFF_Z = EX_W1_BYTES;
constexpr int EX_OFF_XP = EX_OFF_Z + EX_ZSTAGES * EX_Z_BYTES;
constexpr int EX_OFF_W = EX_OFF_XP + EX_ZSTAGES * EX_DH * 4;
constexpr int EX_OFF_HACC = EX_OFF_W + EX_ZSTAGES * EX_ROWS * 4;   // [4 quarters][512] partials
constexpr int EX_OFF_DOTP = EX_OFF_HACC + 4 * EX_DH * 4;
constexpr int EX_OFF_CTL = EX_OFF_DOTP + 2 * EX_ROWS * 4;

struct ExpertCtl {
  uint64_t w1_full;
  uint64_t z_full[EX_ZSTAGES];
  uint64_t z_empty[EX_ZSTAGES];
  uint64_t mma_done[2];
  uint64_t tmem_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr int EX_SMEM_BYTES = EX_OFF_CTL + static_cast<int>(sizeof(ExpertCtl)) + 1024;

struct ExpertFwdArgs {
  const __nv_bfloat16* latents;  // [N, 128]
  const int32_t* ids;            // [T, R]
  const float* w;                // [T, R]
  const float* xp;               // [T, 512]
  __nv_bfloat16* hacc;           // [T, 512]
  float* save_dot;               // [T, R] or null
  int T;
  int R;
  int N;
};

// Byte offset of 16-byte chunk c (0..15) of row r in a 128-row K-major tile
// with 128-byte swizzle (two 64-element K blocks of 16 KB).
__device__ __forceinline__ int ztile_offset(int r, int c) {
  return (c >> 3) * (EX_ROWS * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

__global__ void __launch_bounds__(EX_THREADS, 1)
    k_expert_fwd(const __grid_constant__ CUtensorMap tmW1, ExpertFwdArgs args, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* w1_s = smem;
  uint8_t* z_s = smem + EX_OFF_Z;
  float* xp_s = reinterpret_cast<float*>(smem + EX_OFF_XP);
  float* w_s = reinterpret_cast<float*>(smem + EX_OFF_W);
  float* hacc_s = reinterpret_cast<float*>(smem + EX_OFF_HACC);
  float* dotp_s = reinterpret_cast<float*>(smem + EX_OFF_DOTP);
  ExpertCtl* ctl = reinterpret_cast<ExpertCtl*>(smem + EX_OFF_CTL);
  const int warp = warp_id();
  const int lane = lane_id();
  const int T = args.T, R = args.R;
  const int my_tokens = (T > static_cast<int>(blockIdx.x)) ? (T - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(&ctl->w1_full, 1);
    for (int s = 0; s < EX_ZSTAGES; ++s) {
      mbar_init(&ctl->z_full[s], 64);
      mbar_init(&ctl->z_empty[s], 1 + 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->mma_done[b], 1);
      mbar_init(&ctl->tmem_free[b], 8);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  // zero the A tiles (rows >= R stay zero)
  for (int i = threadIdx.x; i < EX_ZSTAGES * EX_Z_BYTES / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(z_s)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == 2) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort = &ctl->abort;

  if (warp < 2) {
    // ------------------------------------------------------ gather producer
    const int tid = threadIdx.x;  // 0..63
    const int c = tid & 15;
    const int rbase = tid >> 4;
    for (int i = 0; i < my_tokens; ++i) {
      const int t = blockIdx.x + i * gridDim.x;
      const int s = i & 1;
      const uint32_t ph = static_cast<uint32_t>(i >> 1) & 1u;
      if (!mbar_wait(&ctl->z_empty[s], ph ^ 1u, abort, err, 21)) break;
      uint8_t* zt = z_s + s * EX_Z_BYTES;
      const int32_t* idrow = args.ids + static_cast<int64_t>(t) * R;
      for (int j = 0; j < EX_ROWS / 4; ++j) {
        const int r = rbase + 4 * j;
        if (r < R) {
          int id = __ldg(idrow + r);
          if (id < 0 || id >= args.N) {
            record_error(err, ETHOS_ERR_ID_OUT_OF_RANGE);
            id = 0;
          }
          cp_async_16(zt + ztile_offset(r, c), args.latents + static_cast<int64_t>(id) * EX_DL + c * 8);
        }
      }
      const char* xsrc = reinterpret_cast<const char*>(args.xp + static_cast<int64_t>(t) * EX_DH);
      char* xdst = reinterpret_cast<char*>(xp_s + s * EX_DH);
      cp_async_16(xdst + 16 * tid, xsrc + 16 * tid);
      cp_async_16(xdst + 16 * (tid + 64), xsrc + 16 * (tid + 64));
      if (tid < R / 4) {
        cp_async_16(reinterpret_cast<char*>(w_s + s * EX_ROWS) + 16 * tid,
                    reinterpret_cast<const char*>(args.w + static_cast<int64_t>(t) * R) + 16 * tid);
      }
      cp_async_commit_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&ctl->z_full[s]);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true;
      tma_prefetch_desc(&tmW1);
      mbar_arrive_expect_tx(&ctl->w1_full, EX_W1_BYTES);
      for (int kb = 0; kb < 2; ++kb)
        for (int rb = 0; rb < 2; ++rb)
          tma_load_2d(w1_s + kb * (EX_DH * 128) + rb * (256 * 128), &tmW1, &ctl->w1_full, kb * 64, rb * 256);
      if (!mbar_wait(&ctl->w1_full, 0, abort, err, 22)) {
        ok = false;
        mbar_wait(&ctl->w1_full, 0, nullptr, err, 27);  // drain the W1 copy
      }
      const uint32_t idesc = umma_idesc_bf16_f32(128, 256);
      const uint32_t w1_base = smem_u32(w1_s);
      for (int i = 0; ok && i < my_tokens; ++i) {
        const int s = i & 1;
        const uint32_t ph = static_cast<uint32_t>(i >> 1) & 1u;
        if (!mbar_wait(&ctl->z_full[s], ph, abort, err, 23)) break;
        tc_fence_after();
        const uint32_t z_base = smem_u32(z_s + s * EX_Z_BYTES);
        for (int nh = 0; nh < 2; ++nh) {
          if (!mbar_wait(&ctl->tmem_free[nh], (static_cast<uint32_t>(i) & 1u) ^ 1u, abort, err, 24)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < EX_DL / 16; ++k) {
            const int kb = k >> 2, kk = k & 3;
            const uint64_t ad = umma_desc_sw128(z_base + kb * (EX_ROWS * 128) + kk * 32);
            const uint64_t bd = umma_desc_sw128(w1_base + kb * (EX_DH * 128) + nh * (256 * 128) + kk * 32);
            umma_bf16(tmem + nh * 256, ad, bd, idesc, k > 0 ? 1u : 0u);
          }
          umma_commit(&ctl->mma_done[nh]);
        }
        if (!ok) break;
        umma_commit(&ctl->z_empty[s]);
      }
      if (!ok || *abort) {
        umma_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr, err, 28);
      }
    }
  } else if (warp >= 4) {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int g = (warp - 4) >> 2;
    const int r = q * 32 + lane;
    const int etid = (warp - 4) * 32 + lane;  // 0..255
    const bool valid = r < R;
    bool ok = true;
    for (int i = 0; i < my_tokens; ++i) {
      const int t = blockIdx.x + i * gridDim.x;
      const int s = i & 1;
      const uint32_t ph = static_cast<uint32_t>(i >> 1) & 1u;
      const float* xps = xp_s + s * EX_DH;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&ctl->z_full[s], ph, abort, err, 25));
      // pass 1: h = gelu(pre) in place, dot = h . xp
      float dot = 0.f;
      for (int nh = 0; nh < 2; ++nh) {
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&ctl->mma_done[nh], static_cast<uint32_t>(i) & 1u, abort,
                                                        err, 26));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          const int c = nh * 8 + cc * 2 + g;
          float v[32];
          const uint32_t ta = tmem_addr(tmem, q * 32, c * 32);
          tmem_ld32(ta, v);
          const float4* x4 = reinterpret_cast<const float4*>(xps + c * 32);
#pragma unroll
          for (int e4 = 0; e4 < 8; ++e4) {
            const float4 xv = x4[e4];
            float hv;
            hv = gelu_erf(v[4 * e4 + 0]); dot = fmaf(hv, xv.x, dot); v[4 * e4 + 0] = hv;
            hv = gelu_erf(v[4 * e4 + 1]); dot = fmaf(hv, xv.y, dot); v[4 * e4 + 1] = hv;
            hv = gelu_erf(v[4 * e4 + 2]); dot = fmaf(hv, xv.z, dot); v[4 * e4 + 2] = hv;
            hv = gelu_erf(v[4 * e4 + 3]); dot = fmaf(hv, xv.w, dot); v[4 * e4 + 3] = hv;
          }
          tmem_st32(ta, v);
        }
      }
      if (ok) tmem_wait_st();
      dotp_s[g * EX_ROWS + r] = dot;
      named_bar_sync(1, 256);
      dot = dotp_s[r] + dotp_s[EX_ROWS + r];
      const float a = valid ? gelu_erf(dot) * w_s[s * EX_ROWS + r] : 0.f;
      if (args.save_dot != nullptr && g == 0 && valid) args.save_dot[static_cast<int64_t>(t) * R + r] = dot;
      // pass 2: hacc[j] = sum_r a_r h_r[j]
      for (int nh = 0; ok && nh < 2; ++nh) {
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          const int c = nh * 8 + cc * 2 + g;
          float v[32];
          tmem_ld32(tmem_addr(tmem, q * 32, c * 32), v);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = valid ? a * v[e] : 0.f;
          // column sums of this warp's 32 rows; quarters are combined in a
          // fixed order below, so the result is deterministic
          hacc_s[q * EX_DH + c * 32 + lane] = warp_transpose_reduce32(v, lane);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->tmem_free[nh]);
      }
      if (lane == 0) mbar_arrive(&ctl->z_empty[s]);
      named_bar_sync(1, 256);
      {
        const int j = etid * 2;
        const float2 p0 = *reinterpret_cast<const float2*>(hacc_s + j);
        const float2 p1 = *reinterpret_cast<const float2*>(hacc_s + EX_DH + j);
        const float2 p2 = *reinterpret_cast<const float2*>(hacc_s + 2 * EX_DH + j);
        const float2 p3 = *reinterpret_cast<const float2*>(hacc_s + 3 * EX_DH + j);
        const float h0 = (p0.x + p1.x) + (p2.x + p3.x);
        const float h1 = (p0.y + p1.y) + (p2.y + p3.y);
        *reinterpret_cast<uint32_t*>(args.hacc + static_cast<int64_t>(t) * EX_DH + j) = pack_bf16x2(h0, h1);
      }
    }
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace ethos
