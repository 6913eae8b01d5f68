// Pass-2 dZ kernel in the transposed orientation (training path), sm_100a.
//
// The CTA pair computes both views' logit tiles with the vocabulary on the MMA's M side and
// the token rows on its N side: M = 256 lm_head rows (128 per CTA, its TMEM lanes), N = 128
// token rows (each CTA loads 64 of them: the pair splits B), K = H.  Against the row-major
// orientation (M = token rows of both views, N = 128 vocab) the operand that appears twice --
// the two views' hidden rows -- is the split one, so a k-block costs 16 KB of W plus 2 x 8 KB
// of rows per 512 MMA cycles instead of 2 x 16 KB of rows plus 8 KB of W.  With H <= 576 the
// CTA's 128 W rows (up to 9 k-blocks, 144 KB) stay resident for a unit and only the rows
// stream (16 KB per 512 MMA cycles, pass 1's ratio); the resident block is released k-block
// by k-block to the next vocab tile's rows.
//
// Output: dZ^T [vocab chunk, N] bf16 (row stride ld_n), which the GEMM reads K-major for
// dW = dZ^T h_s and MN-major for dH = dZ W; it leaves as one 32 x 32 TMA store per warp and
// 32-column chunk through a 2 KB staging buffer (64-byte swizzle).  The KL cross term
// sum_v p_v (u_t - u_s) is a sum over TMEM lanes here: each warp reduces a 32-column chunk
// across its lanes with a butterfly // transpose-reduction (31 shuffles), the four lane quarters meet in shared memory, and each
// epilogue thread owns 16 columns of every row tile of a unit, whose partials it accumulates
// in registers over the unit's vocabulary tiles -- one partial row per (unit vocab group, CTA).
#pragma once
#include "klg_kernels.cuh"

namespace klg {

constexpr int DZT_BN = 128;                             // token rows per tile
constexpr int DZT_W_BYTES = TILE_128x64;                // this CTA's 128 W rows x 64
constexpr int DZT_H_BYTES = (DZT_BN / 2) * BK * 2;      // this CTA's 64 token rows x 64, one view (8 KB)
constexpr int DZT_MAX_KB = 9;                           // W resident up to H = 576
constexpr int DZT_EPI_WARPS = 8;                        // lane quarter x column half
constexpr int DZT_PW = EPI_WARP0 + DZT_EPI_WARPS;       // first extra producer warp
#ifndef KLG_DZT_PROD
#define KLG_DZT_PROD 2
#endif
constexpr int DZT_PROD = KLG_DZT_PROD;                  // producer warps after the epilogue
constexpr int DZT_THREADS = 32 * (DZT_PW + DZT_PROD);   // + warp 0 (W loader / producer), warp 1 (MMA)
constexpr int DZT_STG_BYTES = 32 * 32 * 2;              // per warp: 32 W rows x 32 token rows bf16 (store staging)
constexpr int DZT_XQ_BYTES = 2 * 4 * DZT_BN * 4;        // cross-term partials [tile parity][lane quarter][column]
constexpr int DZT_BAR_BYTES = 512;
constexpr int DZT_RPU_MAX = 8;                          // row tiles per unit (registers of each owner thread)
template <bool RES>
struct DztCfg {
  static constexpr int A_REGION = RES ? DZT_MAX_KB * DZT_W_BYTES : 0;
  static constexpr int STAGE_BYTES = (RES ? 0 : DZT_W_BYTES) + 2 * DZT_H_BYTES;
  static constexpr int FIXED = 1024 + A_REGION + DZT_EPI_WARPS * DZT_STG_BYTES + DZT_XQ_BYTES + DZT_BAR_BYTES;
  static constexpr int STAGES_RAW = (227 * 1024 - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = FIXED + STAGES * STAGE_BYTES;
  static constexpr int NPROD = RES ? DZT_PROD : DZT_PROD + 1;   // streamed: warp 0 produces too
};

struct DztArgs {
  int n_rows;        // N token rows
  int v_begin;       // first W row of this chunk
  int v_count;       // W rows in the chunk
  int n_vp;          // ceil(v_count / 256): vocab pair tiles
  int n_rt;          // ceil(N / 128): row tiles
  int g;             // vocab pair tiles per unit
  int rpu;           // row tiles per unit (<= DZT_RPU_MAX)
  int n_vg;          // ceil(n_vp / g)
  int n_units;       // n_vg * ceil(n_rt / rpu)
  int n_kb;          // ceil(H / 64)
  float scale_log2;  // log2(e) / T
  const float* lse;      // [2][N] log2-domain log-sum-exp (student, teacher)
  const uint8_t* mask;   // [N]
  const float* count;    // device scalar: number of valid rows (global)
  const float* grad;     // device scalar: upstream gradient, or nullptr for 1
  float inv_temp;
  float* a_parts;        // [.][N] cross-term partials, row a_part_base + vg * 2 + CTA rank
  int a_part_base;
};

// Units are (vocab group, row group), numbered row-group-major: the pairs running at the same
// time stream the same token rows (from L2) against different W tiles.
__device__ __forceinline__ void dzt_unit(const DztArgs& a, int u, int& vg, int& vp0, int& vp1, int& rt0, int& rt1) {
  const int rg = u / a.n_vg;
  vg = u - rg * a.n_vg;
  vp0 = vg * a.g;
  vp1 = min(vp0 + a.g, a.n_vp);
  rt0 = rg * a.rpu;
  rt1 = min(rt0 + a.rpu, a.n_rt);
}

// AND of `p` over the eight epilogue warps (named barrier 1): they agree on whether a tile's
// wait succeeded, so none of them stays behind at the barrier of a tile the others skipped.
__device__ __forceinline__ bool epi_all(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\t"
      "setp.ne.u32 a, %1, 0;\n\t"
      "bar.red.and.pred b, 1, 256, a;\n\t"
      "selp.u32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

// Butterfly transpose-reduction: v[j] of lane l -> lane l holds sum over the 32 lanes of v[l].
__device__ __forceinline__ float lane_transpose_sum(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

template <bool RES>
__global__ void __launch_bounds__(DZT_THREADS, 1)
dzt_pair_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_hs,
                const __grid_constant__ CUtensorMap map_ht, const __grid_constant__ CUtensorMap map_out,
                const DztArgs a) {
  using Cfg = DztCfg<RES>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int STAGE_BYTES = Cfg::STAGE_BYTES;
  constexpr int NPROD = Cfg::NPROD;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t wbase = smem_u32(smem);                                  // resident W (RES)
  const uint32_t sbase = wbase + Cfg::A_REGION;                           // stage ring
  const uint32_t stg0 = sbase + STAGES * STAGE_BYTES;                     // per-warp store staging
  float* xq = reinterpret_cast<float*>(smem + Cfg::A_REGION + STAGES * STAGE_BYTES + DZT_EPI_WARPS * DZT_STG_BYTES);
  const uint32_t bar0 = stg0 + DZT_EPI_WARPS * DZT_STG_BYTES + DZT_XQ_BYTES;
  const uint32_t full0 = bar0;
  const uint32_t empty0 = bar0 + 8u * STAGES;
  const uint32_t tfull0 = bar0 + 16u * STAGES;
  const uint32_t tempty0 = tfull0 + 16u;
  const uint32_t done_bar = tempty0 + 16u;
  const uint32_t wfull0 = done_bar + 8u;                // RES [DZT_MAX_KB]: leader, both CTAs' W bytes
  const uint32_t wempty0 = wfull0 + 8u * DZT_MAX_KB;    // RES [DZT_MAX_KB]: each CTA
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8u * s, 2);
      mbar_init(empty0 + 8u * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8u * b, 1);
      mbar_init(tempty0 + 8u * b, 2 * DZT_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    if (RES) {
      for (int kb = 0; kb < DZT_MAX_KB; ++kb) {
        mbar_init(wfull0 + 8u * kb, 2);
        mbar_init(wempty0 + 8u * kb, 1);
      }
    }
    fence_mbar_init();
    tma_prefetch(&map_w);
    tma_prefetch(&map_hs);
    tma_prefetch(&map_ht);
    tma_prefetch(&map_out);
  }
  if (warp == 1) tmem_alloc_pair(smem_u32(&tmem_slot), DUAL_TMEM_COLS);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_enter();   // inputs of this launch are complete from here on
  volatile int* abort_p = &abort_flag;
  const uint32_t lead_full0 = mapa_shared(full0, 0);
  const uint32_t lead_tempty0 = mapa_shared(tempty0, 0);
  const uint32_t lead_wfull0 = mapa_shared(wfull0, 0);
  const uint32_t peer_empty0 = mapa_shared(empty0, 1);
  const uint32_t peer_tfull0 = mapa_shared(tfull0, 1);
  const uint32_t peer_wempty0 = mapa_shared(wempty0, 1);

  if (RES && warp == 0) {
    // ------------------------------------------------------------ resident W loader (both CTAs, whole warp)
    // k-block kb of a vocab tile's W rows is loaded once the previous tile's last row tile has
    // retired its MMAs on kb (wempty), so the next tile's rows land while that one finishes.
    int seq = -1, kb_loaded = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int vg, vp0, vp1, rt0, rt1;
      dzt_unit(a, u, vg, vp0, vp1, rt0, rt1);
      for (int vp = vp0; ok && vp < vp1; ++vp) {
        ++seq;
        kb_loaded = 0;
        const int wrow = a.v_begin + vp * 256 + (int)rank * 128;
        for (int kb = 0; kb < a.n_kb; ++kb) {
          if (!warp_wait(wempty0 + 8u * kb, (uint32_t)(seq & 1) ^ 1u, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (elect_one()) {
            if (leader) mbar_arrive_expect_tx(wfull0 + 8u * kb, 2 * DZT_W_BYTES);
            tma_load_2d_pair(wbase + kb * DZT_W_BYTES, &map_w, lead_wfull0 + 8u * kb, kb * BK, wrow);
            if (!leader) mbar_arrive_cluster(lead_wfull0 + 8u * kb);
          }
          __syncwarp();
          kb_loaded = kb + 1;
        }
      }
    }
    if (leader) {   // every resident load issued has landed (both CTAs' bytes count on the leader)
      for (int kb = 0; kb < a.n_kb; ++kb) {
        const int last = kb < kb_loaded ? seq : seq - 1;
        if (last >= 0) mbar_wait_drain(wfull0 + 8u * kb, (uint32_t)(last & 1));
      }
    }
  } else if (warp == 0 || warp >= DZT_PW) {
    // ------------------------------------------------------------ streaming producers (both CTAs, whole warp)
    // per (vocab tile, row tile, k-block): this CTA's 64 token rows of both views [+ its 128 W
    // rows when W is not resident]; stage s belongs to producer s % NPROD
    const int prod = RES ? warp - DZT_PW : (warp == 0 ? 0 : warp - DZT_PW + 1);
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int vg, vp0, vp1, rt0, rt1;
      dzt_unit(a, u, vg, vp0, vp1, rt0, rt1);
      for (int vp = vp0; ok && vp < vp1; ++vp) {
        const int wrow = a.v_begin + vp * 256 + (int)rank * 128;
        for (int rt = rt0; ok && rt < rt1; ++rt) {
          const int hrow = rt * DZT_BN + (int)rank * (DZT_BN / 2);
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (stage % NPROD == prod) {
              if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
              if (elect_one()) {
                const uint32_t sa = sbase + stage * STAGE_BYTES;
                const uint32_t fb = lead_full0 + 8u * stage;
                if (leader) mbar_arrive_expect_tx(full0 + 8u * stage, 2 * STAGE_BYTES);
                uint32_t off = 0;
                if (!RES) {
                  tma_load_2d_pair(sa, &map_w, fb, kb * BK, wrow);
                  off = DZT_W_BYTES;
                }
                tma_load_2d_pair(sa + off, &map_hs, fb, kb * BK, hrow);
                tma_load_2d_pair(sa + off + DZT_H_BYTES, &map_ht, fb, kb * BK, hrow);
                if (!leader) mbar_arrive_cluster(fb);
              }
              __syncwarp();
            }
            ++issued;
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
      }
    }
    if (leader && prod == 0) drain_loads<STAGES>(full0, stage, phase, issued);
  } else if (warp == 1) {
    if (leader) {
      // ---------------------------------------------------------- pair MMA issuer (leader, whole warp)
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, DZT_BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      int seq = -1;
      bool ok = true;
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int vg, vp0, vp1, rt0, rt1;
        dzt_unit(a, u, vg, vp0, vp1, rt0, rt1);
        for (int vp = vp0; ok && vp < vp1; ++vp) {
          ++seq;
          for (int rt = rt0; ok && rt < rt1; ++rt, ++tcount) {
            const bool first = rt == rt0, last = rt == rt1 - 1;
            const int buf = tcount & 1;
            const uint32_t tph = (tcount >> 1) & 1;
            if (!warp_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_s = tmem + buf * 256;
            const uint32_t d_t = d_s + 128;
            for (int kb = 0; ok && kb < a.n_kb; ++kb) {
              if (RES && first) {   // this vocab tile's W k-block has landed in both CTAs
                if (!warp_wait(wfull0 + 8u * kb, (uint32_t)(seq & 1), abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
                tc_fence_after();
              }
              if (!warp_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
              tc_fence_after();
              if (elect_one()) {
                const uint32_t sa = sbase + stage * STAGE_BYTES;
                const uint32_t wa = RES ? wbase + kb * DZT_W_BYTES : sa;
                const uint32_t hs_t = RES ? sa : sa + DZT_W_BYTES;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                  const uint64_t adesc = desc_kmajor(wa, k);
                  const uint32_t acc = (kb | k) != 0;
                  mma_bf16_pair(d_s, adesc, desc_kmajor(hs_t, k), idesc, acc);
                  mma_bf16_pair(d_t, adesc, desc_kmajor(hs_t + DZT_H_BYTES, k), idesc, acc);
                }
                mma_commit_pair(empty0 + 8u * stage);
                mma_commit_pair(peer_empty0 + 8u * stage);
              }
              __syncwarp();
              if (++stage == STAGES) { stage = 0; phase ^= 1; }
              if (RES && last && elect_one()) {   // the tile's MMAs on W k-block kb are issued: release it
                mma_commit_pair(wempty0 + 8u * kb);
                mma_commit_pair(peer_wempty0 + 8u * kb);
              }
              __syncwarp();
            }
            if (ok && elect_one()) {
              mma_commit_pair(tfull0 + 8u * buf);
              mma_commit_pair(peer_tfull0 + 8u * buf);
            }
            __syncwarp();
          }
        }
      }
      if (elect_one()) mma_commit_pair(done_bar);
      __syncwarp();
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    // warp (q, h): TMEM lane quarter q (32 W rows), token-row half h of the tile (64 columns)
    const int q = warp & 3;
    const int ew = warp - EPI_WARP0;
    const int h = ew >> 2;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 64);
    const uint32_t stg = stg0 + (uint32_t)ew * DZT_STG_BYTES;
    const uint32_t swz = (uint32_t)((lane >> 1) & 3);   // 64-byte swizzle of the staging rows
    const uint64_t pol = l2_evict_first_policy();       // dZ^T is streamed out once, read by the GEMM
    const float cnt = *a.count;
    const float gsc = a.grad ? *a.grad : 1.0f;
    const float cscale = cnt > 0.f ? gsc / cnt * a.inv_temp : 0.f;
    int tcount = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int vg, vp0, vp1, rt0, rt1;
      dzt_unit(a, u, vg, vp0, vp1, rt0, rt1);
      float acc[DZT_RPU_MAX];
#pragma unroll
      for (int i = 0; i < DZT_RPU_MAX; ++i) acc[i] = 0.f;
      for (int vp = vp0; ok && vp < vp1; ++vp) {
        const int vrow = vp * 256 + (int)rank * 128 + q * 32;   // chunk-relative W row of lane 0
        // W rows past the chunk (its width need not be a multiple of 256) belong to the next
        // chunk: their cross terms are that chunk's, their dZ^T rows are not stored
        const float vmask = vrow + lane < a.v_count ? 1.f : 0.f;
        for (int rt = rt0; rt < rt1; ++rt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          // the row constants of this lane's token rows (one per chunk), fetched before the wait
          float Ls[2], Lt[2], cf[2];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int r = rt * DZT_BN + h * 64 + c * 32 + lane;
            const bool in = r < a.n_rows;
            Ls[c] = in ? a.lse[r] : 0.f;
            Lt[c] = in ? a.lse[a.n_rows + r] : 0.f;
            cf[c] = (in && a.mask[r]) ? cscale : 0.f;
          }
          const bool got = mbar_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE);
          const int par = tcount & 1;
          float* xqp = xq + par * 4 * DZT_BN;
          if (got) {
            tc_fence_after();
            const uint32_t tbase = lane_addr + buf * 256;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int col0 = h * 64 + c * 32;            // first tile column of the chunk
              uint32_t bs[32], bt[32];
              tmem_ld32_raw(tbase + c * 32, bs);
              tmem_ld32_raw(tbase + 128 + c * 32, bt);
              tmem_wait_ld_regs(bs, bt);
              uint32_t pk[16];
              float x[32];
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float Ls0 = __shfl_sync(0xffffffffu, Ls[c], j), Ls1 = __shfl_sync(0xffffffffu, Ls[c], j + 1);
                const float Lt0 = __shfl_sync(0xffffffffu, Lt[c], j), Lt1 = __shfl_sync(0xffffffffu, Lt[c], j + 1);
                const float c0 = __shfl_sync(0xffffffffu, cf[c], j), c1 = __shfl_sync(0xffffffffu, cf[c], j + 1);
                const float zs0 = __uint_as_float(bs[j]), zs1 = __uint_as_float(bs[j + 1]);
                const float zt0 = __uint_as_float(bt[j]), zt1 = __uint_as_float(bt[j + 1]);
                const float q0 = ex2(fmaf(zs0, a.scale_log2, -Ls0));
                const float q1 = ex2(fmaf(zs1, a.scale_log2, -Ls1));
                const float p0 = ex2(fmaf(zt0, a.scale_log2, -Lt0));
                const float p1 = ex2(fmaf(zt1, a.scale_log2, -Lt1));
                pk[j / 2] = pack_bf16x2(c0 * (q0 - p0), c1 * (q1 - p1));
                x[j] = vmask * p0 * (zt0 - zs0);
                x[j + 1] = vmask * p1 * (zt1 - zs1);
              }
              // dZ^T rows vrow .. +31 x token columns rt * 128 + col0 .. +31: one 32 x 32 TMA store;
              // the staging buffer is free once the previous chunk's store has read it
              if (lane == 0) bulk_wait_read0();
              __syncwarp();
              const uint32_t rowp = stg + (uint32_t)lane * 64u;
#pragma unroll
              for (int k = 0; k < 4; ++k)
                st_shared_v4(rowp + (((uint32_t)k ^ swz) << 4), pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
              fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                const int x0 = rt * DZT_BN + col0;
                if (vrow < a.v_count && x0 < a.n_rows) tma_store_2d_hint(&map_out, stg, x0, vrow, pol);
                bulk_commit();
              }
              // this warp's 32 W rows' part of the cross term of the chunk's 32 token rows
              xqp[q * DZT_BN + col0 + lane] = lane_transpose_sum(x);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if (leader) mbar_arrive(tempty0 + 8u * buf);
              else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
            }
          }
          // all eight warps agree the tile was there (and have written its partials)
          if (!epi_all(got)) {
            ok = false;
            break;
          }
          // each warp owns 16 columns of every row tile: the four lane quarters' partials
          if (lane < 16) {
            const int col = ew * 16 + lane;
            const float s = (xqp[col] + xqp[DZT_BN + col]) + (xqp[2 * DZT_BN + col] + xqp[3 * DZT_BN + col]);
#pragma unroll
            for (int i = 0; i < DZT_RPU_MAX; ++i)
              if (i == rt - rt0) acc[i] += s;
          }
        }
      }
      if (ok && lane < 16 && a.a_parts) {
        float* dst = a.a_parts + (size_t)(a.a_part_base + vg * 2 + (int)rank) * a.n_rows;
#pragma unroll
        for (int i = 0; i < DZT_RPU_MAX; ++i) {
          const int row = (rt0 + i) * DZT_BN + ew * 16 + lane;
          if (rt0 + i < rt1 && row < a.n_rows) dst[row] = acc[i] * a.scale_log2;
        }
      }
    }
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, DUAL_TMEM_COLS);
}

}  // namespace klg
