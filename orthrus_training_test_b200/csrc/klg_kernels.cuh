// sm_100a kernels of the fused KL-GEMM distillation loss.
//
// Notation: N rows (student/teacher pairs), H hidden, V vocab, W = lm_head [V, H].
// Logits are z = h W^T / T.  All softmax arithmetic runs in the log2 domain:
// u = z * log2(e) / T, so exp(z - m) = 2^(u - m2).
//
//  dual_kernel<STATS>  pass 1: per (row tile, vocab range) unit, both views'
//                      logit tiles 128 x 128 via tcgen05.mma into TMEM, epilogue
//                      keeps per-row online (m_s, S_s, m_t, S_t, A) and writes
//                      one partial record per unit.
//  dual_kernel<DZ>     pass 2: recomputes both views' logit tiles for one vocab
//                      chunk and writes dZ = g/n * valid * (q - p) / T as bf16.
//  gemm_kernel         D (+)= A * B with K-major or MN-major bf16 operands, fp32
//                      out: dH += dZ W_chunk and dW_chunk = dZ^T h_s.
//
// Warp roles (all kernels): warp 0 issues TMA loads, warp 1 allocates TMEM and
// issues tcgen05.mma from one thread, warps 2..5 are the epilogue (one TMEM lane,
// i.e. one output row, per thread).  Shared-memory stages are recycled through
// full/empty mbarriers; the two TMEM accumulator buffers through tmem_full /
// tmem_empty so the epilogue of tile j overlaps the MMAs of tile j+1.
#pragma once
#include "klg_ptx.cuh"

namespace klg {

constexpr int BM = 128;                     // rows per tile (TMEM lanes)
constexpr int BK = 64;                      // bf16 elements per k-block (one 128 B swizzle row)
constexpr int TILE_128x64 = BM * BK * 2;    // 16 KB
constexpr int NUM_THREADS = 192;
constexpr int EPI_WARP0 = 2;
constexpr float NEG_BIG = -1.0e30f;

// =====================================================================================
// dual-view kernel
// =====================================================================================
constexpr int DUAL_BN = 128;
constexpr int DUAL_STAGES = 4;
constexpr int DUAL_STAGE_BYTES = 3 * TILE_128x64;  // A_s | A_t | B
constexpr int DUAL_TMEM_COLS = 512;                // 2 buffers x (Z_s 128 | Z_t 128)
constexpr int DUAL_SMEM = 1024 + DUAL_STAGES * DUAL_STAGE_BYTES + 256;

enum { MODE_STATS = 0, MODE_DZ = 1 };

struct DualArgs {
  int n_rows;       // N
  int v_begin;      // first W row of this launch
  int v_count;      // W rows covered by this launch
  int n_rt;         // ceil(N / 128)
  int n_vt;         // ceil(v_count / 128)
  int vt_per_unit;  // vocab tiles per work unit
  int n_units;      // n_rt * ceil(n_vt / vt_per_unit)
  int n_kb;         // ceil(H / 64)
  float scale_log2; // log2(e) / T
  // MODE_STATS
  float* partials;  // [n_uv][5][N]
  // MODE_DZ
  const float* lse;      // [2][N] log2-domain log-sum-exp (student, teacher)
  const uint8_t* mask;   // [N]
  const float* count;    // device scalar: number of valid rows (global)
  const float* grad;     // device scalar: upstream gradient, or nullptr for 1
  float inv_temp;
  __nv_bfloat16* dz;     // [N][ld_dz], column j = W row v_begin + j
  int ld_dz;
};

__device__ __forceinline__ void dual_unit(const DualArgs& a, int u, int& rt, int& uv, int& vt0, int& vt1) {
  rt = u % a.n_rt;
  uv = u / a.n_rt;
  vt0 = uv * a.vt_per_unit;
  vt1 = min(vt0 + a.vt_per_unit, a.n_vt);
}

// Bounded wait used only while draining at kernel exit (ignores the abort flag).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > KLG_WAIT_CYCLES) {
      atomicOr(&g_status, KLG_STATUS_TIMEOUT_DRAIN);
      return false;
    }
  }
  return true;
}

// Waits until the last loads issued into each stage have landed (TMA copies
// complete on their own; this keeps them from outliving the CTA on abort).
template <int STAGES>
__device__ __forceinline__ void drain_loads(uint32_t full0, int stage, uint32_t phase, long long issued) {
  const int n = issued < STAGES ? (int)issued : STAGES;
  for (int j = 0; j < n; ++j) {
    if (stage == 0) { stage = STAGES; phase ^= 1; }
    --stage;
    mbar_wait_drain(full0 + 8u * stage, phase);
  }
}

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
dual_kernel(const __grid_constant__ CUtensorMap map_hs, const __grid_constant__ CUtensorMap map_ht,
            const __grid_constant__ CUtensorMap map_w, const DualArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + DUAL_STAGES * DUAL_STAGE_BYTES;
  const uint32_t full0 = bar0;                          // [STAGES]
  const uint32_t empty0 = bar0 + 8u * DUAL_STAGES;      // [STAGES]
  const uint32_t tfull0 = bar0 + 16u * DUAL_STAGES;     // [2]
  const uint32_t tempty0 = tfull0 + 16u;                // [2]
  const uint32_t done_bar = tempty0 + 16u;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < DUAL_STAGES; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8u * b, 1);
      mbar_init(tempty0 + 8u * b, 4 * 32);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch(&map_hs);
    tma_prefetch(&map_ht);
    tma_prefetch(&map_w);
  }
  if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), DUAL_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < a.n_units; u += gridDim.x) {
        int rt, uv, vt0, vt1;
        dual_unit(a, u, rt, uv, vt0, vt1);
        for (int vt = vt0; ok && vt < vt1; ++vt) {
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!mbar_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
            const uint32_t sb = sbase + stage * DUAL_STAGE_BYTES;
            const uint32_t fb = full0 + 8u * stage;
            mbar_arrive_expect_tx(fb, DUAL_STAGE_BYTES);
            tma_load_2d(sb, &map_hs, fb, kb * BK, rt * BM);
            tma_load_2d(sb + TILE_128x64, &map_ht, fb, kb * BK, rt * BM);
            tma_load_2d(sb + 2 * TILE_128x64, &map_w, fb, kb * BK, a.v_begin + vt * DUAL_BN);
            ++issued;
            if (++stage == DUAL_STAGES) { stage = 0; phase ^= 1; }
          }
        }
      }
      drain_loads<DUAL_STAGES>(full0, stage, phase, issued);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = make_idesc_bf16(BM, DUAL_BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < a.n_units; u += gridDim.x) {
        int rt, uv, vt0, vt1;
        dual_unit(a, u, rt, uv, vt0, vt1);
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          if (!mbar_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_s = tmem + buf * 256;
          const uint32_t d_t = d_s + 128;
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!mbar_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sb = sbase + stage * DUAL_STAGE_BYTES;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t bdesc = desc_kmajor(sb + 2 * TILE_128x64, k);
              const uint32_t acc = (kb | k) != 0;
              mma_bf16(d_s, desc_kmajor(sb, k), bdesc, idesc, acc);
              mma_bf16(d_t, desc_kmajor(sb + TILE_128x64, k), bdesc, idesc, acc);
            }
            mma_commit(empty0 + 8u * stage);
            if (++stage == DUAL_STAGES) { stage = 0; phase ^= 1; }
          }
          if (ok) mma_commit(tfull0 + 8u * buf);
        }
      }
      // all issued MMAs must retire before TMEM is released
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int r_in_tile = q * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    int tcount = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < a.n_units; u += gridDim.x) {
      int rt, uv, vt0, vt1;
      dual_unit(a, u, rt, uv, vt0, vt1);
      const int row = rt * BM + r_in_tile;
      const bool row_ok = row < a.n_rows;
      // per-row state
      float ms = NEG_BIG, Ss = 0.f, mt = NEG_BIG, St = 0.f, A = 0.f;  // STATS
      float Ls = 0.f, Lt = 0.f, coef = 0.f;                            // DZ
      if (MODE == MODE_DZ && row_ok) {
        Ls = a.lse[row];
        Lt = a.lse[a.n_rows + row];
        const float cnt = *a.count;
        const float g = a.grad ? *a.grad : 1.0f;
        coef = (a.mask[row] && cnt > 0.f) ? g / cnt * a.inv_temp : 0.f;
      }
      for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        if (!mbar_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DUAL_BN / 32; ++c) {
          float zs[32], zt[32];
          tmem_ld32(lane_addr + buf * 256 + c * 32, zs);
          tmem_ld32(lane_addr + buf * 256 + 128 + c * 32, zt);
          tmem_wait_ld();
          const int col0 = vt * DUAL_BN + c * 32;      // relative to v_begin
          const int nvalid = min(32, a.v_count - col0);
          if (nvalid <= 0) continue;
          if (MODE == MODE_STATS) {
            float cms = -INFINITY, cmt = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const bool v = j < nvalid;
              zs[j] = v ? zs[j] * a.scale_log2 : -INFINITY;
              zt[j] = v ? zt[j] * a.scale_log2 : -INFINITY;
              cms = fmaxf(cms, zs[j]);
              cmt = fmaxf(cmt, zt[j]);
            }
            const float nms = fmaxf(ms, cms);
            const float nmt = fmaxf(mt, cmt);
            const float rs = ex2(ms - nms);
            const float rt_ = ex2(mt - nmt);
            ms = nms;
            mt = nmt;
            float s0 = 0.f, s1 = 0.f, t0 = 0.f, t1 = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              s0 += ex2(zs[j] - ms);
              s1 += ex2(zs[j + 1] - ms);
              const float e0 = ex2(zt[j] - mt);
              const float e1 = ex2(zt[j + 1] - mt);
              t0 += e0;
              t1 += e1;
              a0 = fmaf(e0, (j < nvalid) ? zt[j] - zs[j] : 0.f, a0);
              a1 = fmaf(e1, (j + 1 < nvalid) ? zt[j + 1] - zs[j + 1] : 0.f, a1);
            }
            Ss = fmaf(Ss, rs, s0 + s1);
            St = fmaf(St, rt_, t0 + t1);
            A = fmaf(A, rt_, a0 + a1);
          } else {
            if (!row_ok) continue;
            __nv_bfloat16* dst = a.dz + (size_t)row * a.ld_dz + col0;
            uint32_t pk[16];
            if (coef == 0.f) {
#pragma unroll
              for (int j = 0; j < 16; ++j) pk[j] = 0u;
            } else {
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float q0 = ex2(fmaf(zs[j], a.scale_log2, -Ls));
                const float q1 = ex2(fmaf(zs[j + 1], a.scale_log2, -Ls));
                const float p0 = ex2(fmaf(zt[j], a.scale_log2, -Lt));
                const float p1 = ex2(fmaf(zt[j + 1], a.scale_log2, -Lt));
                pk[j / 2] = pack_bf16x2(coef * (q0 - p0), coef * (q1 - p1));
              }
            }
            if (nvalid == 32) {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 4; ++j) d4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            } else {
              unsigned short* d2 = reinterpret_cast<unsigned short*>(dst);
              for (int j = 0; j < nvalid; ++j) d2[j] = (unsigned short)((pk[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(tempty0 + 8u * buf);
      }
      if (MODE == MODE_STATS && ok && row_ok) {
        float* p = a.partials + (size_t)uv * 5 * a.n_rows + row;
        p[0] = ms;
        p[(size_t)a.n_rows] = Ss;
        p[(size_t)2 * a.n_rows] = mt;
        p[(size_t)3 * a.n_rows] = St;
        p[(size_t)4 * a.n_rows] = A;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, DUAL_TMEM_COLS);
}

// =====================================================================================
// generic GEMM: C[M][Ncol] (+)= A[M][K] * B[K][Ncol], bf16 in, fp32 out
// =====================================================================================
struct GemmArgs {
  int M, Ncol, K;
  int n_mt, n_nt, n_tiles, n_kb;
  float* C;
  int ldc;
  int accumulate;   // 1: C += A*B, 0: C = A*B
  int a_k0, b_k0;   // K coordinate of the first k-block in A's and B's tensor maps
};

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = TILE_128x64;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 192) ? 4 : 6;
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
};

// A_MN: A stored [K][M] (M contiguous), loaded as two 64-wide boxes.
// B_MN: B stored [K][Ncol] (Ncol contiguous), loaded as BN/64 boxes; otherwise
//       B stored [Ncol][K] (K contiguous) and loaded as one 64 x BN box.
template <bool A_MN, bool B_MN, int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, const GemmArgs a) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + STAGES * Cfg::STAGE_BYTES;
  const uint32_t full0 = bar0;
  const uint32_t empty0 = bar0 + 8u * STAGES;
  const uint32_t tfull0 = bar0 + 16u * STAGES;
  const uint32_t tempty0 = tfull0 + 16u;
  const uint32_t done_bar = tempty0 + 16u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8u * b, 1);
      mbar_init(tempty0 + 8u * b, 4 * 32);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
  }
  if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < a.n_tiles; t += gridDim.x) {
        const int mt = t / a.n_nt, nt = t % a.n_nt;
        for (int kb = 0; kb < a.n_kb; ++kb) {
          if (!mbar_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
          const uint32_t sa = sbase + stage * Cfg::STAGE_BYTES;
          const uint32_t sb = sa + Cfg::A_BYTES;
          const uint32_t fb = full0 + 8u * stage;
          mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
          const int ka = a.a_k0 + kb * BK, kbb = a.b_k0 + kb * BK;
          if (A_MN) {
            tma_load_2d(sa, &map_a, fb, mt * BM, ka);
            tma_load_2d(sa + 8192, &map_a, fb, mt * BM + 64, ka);
          } else {
            tma_load_2d(sa, &map_a, fb, ka, mt * BM);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + 8192 * j, &map_b, fb, nt * BN + 64 * j, kbb);
          } else {
            tma_load_2d(sb, &map_b, fb, kbb, nt * BN);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      drain_loads<STAGES>(full0, stage, phase, issued);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < a.n_tiles; t += gridDim.x, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        if (!mbar_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < a.n_kb; ++kb) {
          if (!mbar_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = sbase + stage * Cfg::STAGE_BYTES;
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? desc_mnmajor(sa, k) : desc_kmajor(sa, k);
            const uint64_t bd = B_MN ? desc_mnmajor(sb, k) : desc_kmajor(sb, k);
            mma_bf16(d, ad, bd, idesc, (kb | k) != 0);
          }
          mma_commit(empty0 + 8u * stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(tfull0 + 8u * buf);
      }
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    const int q = warp & 3;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    int tcount = 0;
    for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x, ++tcount) {
      const int mt = t / a.n_nt, nt = t % a.n_nt;
      const int buf = tcount & 1;
      const uint32_t tph = (tcount >> 1) & 1;
      if (!mbar_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
      const bool row_ok = row < a.M;
      float* crow = a.C + (size_t)row * a.ldc;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(lane_addr + buf * BN + c * 32, v);
        tmem_wait_ld();
        const int col0 = nt * BN + c * 32;
        if (!row_ok || col0 >= a.Ncol) continue;
        if (col0 + 32 <= a.Ncol) {
          float4* d4 = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            if (a.accumulate) {
              const float4 old = d4[j];
              o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
            }
            d4[j] = o;
          }
        } else {
          for (int j = 0; j < a.Ncol - col0; ++j) crow[col0 + j] = a.accumulate ? crow[col0 + j] + v[j] : v[j];
        }
      }
      tc_fence_before();
      mbar_arrive(tempty0 + 8u * buf);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

// =====================================================================================
// small kernels
// =====================================================================================

// count = sum(mask), one block, deterministic.
__global__ void count_valid_kernel(const uint8_t* __restrict__ mask, int n, float* __restrict__ count) {
  __shared__ int part[32];
  int c = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) c += mask[i] != 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x < 32) {
    c = (threadIdx.x < (blockDim.x >> 5)) ? part[threadIdx.x] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (threadIdx.x == 0) *count = (float)c;
  }
}

// Online-softmax merge of n_part partial records [n_part][5][N] -> [5][N].
__global__ void merge_kernel(const float* __restrict__ parts, int n_part, int n, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const size_t st = (size_t)n;
  float ms = NEG_BIG, mt = NEG_BIG;
  for (int p = 0; p < n_part; ++p) {
    ms = fmaxf(ms, parts[(size_t)p * 5 * st + i]);
    mt = fmaxf(mt, parts[(size_t)p * 5 * st + 2 * st + i]);
  }
  float Ss = 0.f, St = 0.f, A = 0.f;
  for (int p = 0; p < n_part; ++p) {
    const float* q = parts + (size_t)p * 5 * st + i;
    const float ws = ex2(q[0] - ms);
    const float wt = ex2(q[2 * st] - mt);
    Ss = fmaf(q[st], ws, Ss);
    St = fmaf(q[3 * st], wt, St);
    A = fmaf(q[4 * st], wt, A);
  }
  out[i] = ms;
  out[st + i] = Ss;
  out[2 * st + i] = mt;
  out[3 * st + i] = St;
  out[4 * st + i] = A;
}

// From merged records: lse (log2 domain) [2][N], optional per-row KL (nats),
// and loss = sum(valid * KL) / count.  One block, deterministic tree reduction.
__global__ void finalize_kernel(const float* __restrict__ stats, const uint8_t* __restrict__ mask, int n,
                                const float* __restrict__ count, float* __restrict__ loss,
                                float* __restrict__ lse, float* __restrict__ row_kl) {
  __shared__ float part[32];
  const size_t st = (size_t)n;
  const float ln2 = 0.69314718055994530942f;
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float ms = stats[i], Ss = stats[st + i], mt = stats[2 * st + i], St = stats[3 * st + i], A = stats[4 * st + i];
    const float Ls = ms + __log2f(Ss);
    const float Lt = mt + __log2f(St);
    const float kl = ln2 * (A / St + Ls - Lt);
    if (lse) {
      lse[i] = Ls;
      lse[st + i] = Lt;
    }
    if (row_kl) row_kl[i] = kl;
    if (mask[i]) acc += kl;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = (threadIdx.x < (blockDim.x >> 5)) ? part[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x == 0) {
      const float c = *count;
      *loss = c > 0.f ? acc / c : 0.f;
    }
  }
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = i; j < n; j += stride) out[j] = __float2bfloat16_rn(in[j]);
}

}  // namespace klg
