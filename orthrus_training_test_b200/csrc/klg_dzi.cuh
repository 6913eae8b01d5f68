// Pass-2 dZ kernel with the two views interleaved along the MMA's M side (training path),
// sm_100a.
//
// The row-major dZ kernel (dual_pair_kernel<MODE_DZ>) runs one MMA per view: each CTA loads
// 128 student rows, 128 teacher rows and 64 W rows per k-block -- 40 KB per 512 MMA cycles,
// which the TMA ring cannot keep up with (its tensor pipe idles ~17 % of the time waiting on
// operands).  Here a CTA's 128 MMA rows are 64 token rows x 2 views, interleaved, and one
// N = 256 MMA covers both views: a k-block costs 16 KB of rows plus 16 KB of W (128 rows) per
// 512 MMA cycles, and two TMA copies instead of three.
//
// The interleave comes from one tensor map over both tensors whose view dimension has the
// distance between the two base pointers as its stride (view 0 = the lower address).  TMA reads
// only the two tensors' own rows: every coordinate stays inside the map's extents, and rows past
// N are zero-filled.  Two layouts:
//
//  DZI_G8 (N % 8 == 0): a 4-D map {H, 8 rows, 2 views, N / 8 groups}, box {64, 8, 2, 8}: MMA row
//    16 g + 8 v + r is row r of 8-row group g in view v.  A tcgen05.ld of shape 16x256b gives each
//    thread lanes l and l + 8 of a 16-lane group -- one token row's logits in both views, two
//    adjacent columns per 8 -- so the epilogue works on (student, teacher) pairs in registers, with
//    packed fp32x2 arithmetic: per pair of columns 2 FMA2 for the exponent arguments, 4 ex2, 2 for
//    dZ, 1 bf16x2 convert, 2 for the cross term.
//  DZI_ROW (any N): a 3-D map {H, 2 views, N rows}, box {64, 2, 64}: MMA row 2 r + v.  With the
//    32x32b TMEM shape each thread holds one view of one token row; the lane pair (2r, 2r + 1)
//    swaps half of a 32-column chunk with one shuffle per value.
//
// Either way each warp writes a 16-row x 64-column dZ block per TMA store (two 2 KB staging
// buffers, 128-byte swizzle) and keeps its rows' KL cross term sum_v p_v (u_t - u_s), summed over
// the threads sharing a row at the end of a unit.  Rows whose mask is off (or a batch with no
// valid row) get dZ = 0 without the arithmetic when no row of the warp's half needs it.
#pragma once
#include "klg_kernels.cuh"

namespace klg {

constexpr int DZI_BN = 256;                          // vocab columns per pair tile (128 W rows per CTA)
constexpr int DZI_ROWS = 128;                        // token rows per pair tile (64 per CTA, both views)
constexpr int DZI_A_BYTES = TILE_128x64;             // 64 token rows x 2 views x 64 (16 KB)
constexpr int DZI_B_BYTES = (DZI_BN / 2) * BK * 2;   // 128 W rows x 64 (16 KB)
constexpr int DZI_STAGE_BYTES = DZI_A_BYTES + DZI_B_BYTES;
constexpr int DZI_EPI_WARPS = 8;                     // lane quarter x 128-column half
constexpr int DZI_CSPLIT = 2;                        // cross-term partial rows per unit (column halves)
constexpr int DZI_PW = EPI_WARP0 + DZI_EPI_WARPS;    // first extra producer warp
#ifndef KLG_DZI_PROD
#define KLG_DZI_PROD 2
#endif
constexpr int DZI_PROD = KLG_DZI_PROD;               // producer warps: warp 0 and DZI_PROD - 1 after the epilogue
constexpr int DZI_THREADS = 32 * (DZI_PW + DZI_PROD - 1);
constexpr int DZI_STG_BYTES = 2 * 16 * 128;          // per warp: 2 buffers x (16 token rows x 64 bf16)
constexpr int DZI_STORE_COLS = 64;                   // columns per TMA store box (16 rows high)
constexpr int DZI_FIXED = 1024 + DZI_EPI_WARPS * DZI_STG_BYTES + 256;
constexpr int DZI_STAGES_RAW = (227 * 1024 - DZI_FIXED) / DZI_STAGE_BYTES;
constexpr int DZI_STAGES = DZI_STAGES_RAW > 8 ? 8 : DZI_STAGES_RAW;
constexpr int DZI_SMEM = DZI_FIXED + DZI_STAGES * DZI_STAGE_BYTES;
static_assert(DZI_SMEM <= 227 * 1024, "dzi shared memory");

// layouts of the interleaved rows (template argument of dzi_pair_kernel)
constexpr int DZI_ROW = 0;      // MMA row 2 r + v
constexpr int DZI_G8_S0 = 1;    // MMA row 16 g + 8 v + r, the student rows are view 0
constexpr int DZI_G8_S1 = 2;    // as DZI_G8_S0, the student rows are view 1

struct DziArgs {
  int n_rows;        // N token rows
  int v_begin;       // first W row of this chunk
  int v_count;       // W rows in the chunk
  int n_rt;          // ceil(N / 128): pair row tiles
  int n_vt;          // ceil(v_count / 256): vocab tiles
  int vt_per_unit;   // vocab tiles per work unit
  int n_units;       // n_rt * ceil(n_vt / vt_per_unit)
  int n_kb;          // ceil(H / 64)
  int s_view;        // view index (0 or 1) of the student rows (DZI_ROW; the G8 layouts fix it)
  float scale_log2;  // log2(e) / T
  const float* lse;      // [2][N] log2-domain log-sum-exp (student, teacher)
  const uint8_t* mask;   // [N]
  const float* count;    // device scalar: number of valid rows (global)
  const float* grad;     // device scalar: upstream gradient, or nullptr for 1
  float inv_temp;
  float* a_parts;        // optional [.][N]: cross-term partial rows a_part_base + uv * DZI_CSPLIT + half
  int a_part_base;
  float* partials;       // MODE_STATS: [n_uv * DZI_CSPLIT][5][N] records (m_s, S_s, m_t, S_t, A), log2 units
};

// Units are numbered row-tile-major (the pairs running at the same time share a few row tiles
// in L2 while each sweeps its own vocabulary range).
__device__ __forceinline__ void dzi_unit(const DziArgs& a, int u, int& rt, int& uv, int& vt0, int& vt1) {
  const int n_uv = (a.n_vt + a.vt_per_unit - 1) / a.vt_per_unit;
  rt = u / n_uv;
  uv = u - rt * n_uv;
  vt0 = uv * a.vt_per_unit;
  vt1 = min(vt0 + a.vt_per_unit, a.n_vt);
}

// Per-row constants of the dZ epilogue.  live: the row takes part in the loss (mask set, count
// > 0); coef = g / count / T for live rows, 0 otherwise.
struct DziRow {
  float Ls, Lt, coef;
  bool live;
};
__device__ __forceinline__ DziRow dzi_row(const DziArgs& a, int row) {
  DziRow r{0.f, 0.f, 0.f, false};
  if (row < a.n_rows) {
    r.Ls = a.lse[row];
    r.Lt = a.lse[a.n_rows + row];
    const float cnt = *a.count;
    r.live = a.mask[row] && cnt > 0.f;
    const float g = a.grad ? *a.grad : 1.0f;
    r.coef = r.live ? g / cnt * a.inv_temp : 0.f;
  }
  return r;
}

// G8 epilogue on one 16x256b.x4 load (32 columns): r[4k + 2 SV .. +1] are the student's logits
// at columns 8k + 2 tq + {0, 1}, the other two the teacher's.  pk[k] = bf16x2 dZ of those
// columns; acc (packed pair) += p (z_t - z_s) over the columns below ncol (MASK) or all of them.
template <int SV, bool MASK>
__device__ __forceinline__ void dzi_g8_chunk(const uint32_t (&r)[16], uint64_t sl2, uint64_t nls, uint64_t nlt,
                                             uint64_t coef, int col0, int ncol, uint32_t (&pk)[4], uint64_t& acc) {
  const uint64_t neg1 = f2_pack(-1.f, -1.f);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint64_t zs = f2_pack(__uint_as_float(r[4 * k + 2 * SV]), __uint_as_float(r[4 * k + 2 * SV + 1]));
    const uint64_t zt = f2_pack(__uint_as_float(r[4 * k + 2 - 2 * SV]), __uint_as_float(r[4 * k + 3 - 2 * SV]));
    float as0, as1, at0, at1;
    f2_unpack(f2_fma(zs, sl2, nls), as0, as1);
    f2_unpack(f2_fma(zt, sl2, nlt), at0, at1);
    const float q0 = ex2(as0), q1 = ex2(as1), p0 = ex2(at0), p1 = ex2(at1);
    const uint64_t p = f2_pack(p0, p1);
    float d0, d1;
    f2_unpack(f2_mul(f2_fma(p, neg1, f2_pack(q0, q1)), coef), d0, d1);
    pk[k] = pack_bf16x2(d0, d1);
    const uint64_t dzt = f2_sub(zt, zs);
    if (MASK) {
      const int c = col0 + 8 * k;
      acc = f2_fma(f2_pack(c < ncol ? p0 : 0.f, c + 1 < ncol ? p1 : 0.f), dzt, acc);
    } else {
      acc = f2_fma(p, dzt, acc);
    }
  }
}

// G8 statistics on one 16x256b.x4 load (32 columns, 8 per thread: columns col0 + 8k + {0, 1}):
// the online (m_s, S_s, m_t, S_t, A) update of stats_chunk, A = sum 2^(u_t - m_t) (u_t - u_s),
// with u = z * sl2; columns at or past ncol are left out (MASK).
template <int SV, bool MASK>
__device__ __forceinline__ void dzi_g8_stats(const uint32_t (&r)[16], uint64_t sl2, int col0, int ncol,
                                             float (&st)[5]) {
  float us[8], ut[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint64_t zs = f2_pack(__uint_as_float(r[4 * k + 2 * SV]), __uint_as_float(r[4 * k + 2 * SV + 1]));
    const uint64_t zt = f2_pack(__uint_as_float(r[4 * k + 2 - 2 * SV]), __uint_as_float(r[4 * k + 3 - 2 * SV]));
    f2_unpack(f2_mul(zs, sl2), us[2 * k], us[2 * k + 1]);
    f2_unpack(f2_mul(zt, sl2), ut[2 * k], ut[2 * k + 1]);
    if (MASK) {
#pragma unroll
      for (int e = 0; e < 2; ++e)
        if (col0 + 8 * k + e >= ncol) us[2 * k + e] = ut[2 * k + e] = -INFINITY;
    }
  }
  float cms = us[0], cmt = ut[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) {
    cms = fmaxf(cms, us[j]);
    cmt = fmaxf(cmt, ut[j]);
  }
  const float nms = fmaxf(st[0], cms), nmt = fmaxf(st[2], cmt);
  const float rs = ex2(st[0] - nms), rt = ex2(st[2] - nmt);
  const uint64_t ms2 = f2_pack(nms, nms), mt2 = f2_pack(nmt, nmt);
  uint64_t ss = 0, stt = 0, aa = 0;   // packed (0.f, 0.f)
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint64_t u_s = f2_pack(us[2 * k], us[2 * k + 1]), u_t = f2_pack(ut[2 * k], ut[2 * k + 1]);
    float a0, a1, b0, b1;
    f2_unpack(f2_sub(u_s, ms2), a0, a1);
    f2_unpack(f2_sub(u_t, mt2), b0, b1);
    const uint64_t es = f2_pack(ex2(a0), ex2(a1)), et = f2_pack(ex2(b0), ex2(b1));
    ss = f2_add(ss, es);
    stt = f2_add(stt, et);
    uint64_t d = f2_sub(u_t, u_s);
    if (MASK) {   // left-out columns: e_t = 0 but u_t - u_s is NaN
      float d0, d1;
      f2_unpack(d, d0, d1);
      d = f2_pack(col0 + 8 * k < ncol ? d0 : 0.f, col0 + 8 * k + 1 < ncol ? d1 : 0.f);
    }
    aa = f2_fma(et, d, aa);
  }
  float x0, x1;
  f2_unpack(ss, x0, x1);
  st[1] = fmaf(st[1], rs, x0 + x1);
  f2_unpack(stt, x0, x1);
  st[3] = fmaf(st[3], rt, x0 + x1);
  f2_unpack(aa, x0, x1);
  st[4] = fmaf(st[4], rt, x0 + x1);
  st[0] = nms;
  st[2] = nmt;
}

// Online merge of this thread's record with the one of lane ^ o (same row, other columns).
__device__ __forceinline__ void dzi_stats_merge(float (&st)[5], int o) {
  float q[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) q[i] = __shfl_xor_sync(0xffffffffu, st[i], o);
  const float ms = fmaxf(st[0], q[0]), mt = fmaxf(st[2], q[2]);
  const float a = ex2(st[0] - ms), b = ex2(q[0] - ms), c = ex2(st[2] - mt), d = ex2(q[2] - mt);
  st[1] = fmaf(st[1], a, q[1] * b);
  st[3] = fmaf(st[3], c, q[3] * d);
  st[4] = fmaf(st[4], c, q[4] * d);
  st[0] = ms;
  st[2] = mt;
}

// MODE_DZ: pass 2's dZ chunk and KL cross-term partials.  MODE_STATS (G8 layouts only): the
// single-pass forward's per-unit records (m_s, S_s, m_t, S_t, A) for evaluation.
template <int LAY, int MODE = MODE_DZ>
__global__ void __launch_bounds__(DZI_THREADS, 1)
dzi_pair_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_out, const DziArgs a) {
  constexpr bool G8 = LAY != DZI_ROW;
  constexpr int SV = LAY == DZI_G8_S1 ? 1 : 0;
  static_assert(MODE == MODE_DZ || G8, "the statistics epilogue is built for the 8-row-group layouts");
  constexpr int STAGES = DZI_STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t stg0 = sbase + STAGES * DZI_STAGE_BYTES;   // 1024-aligned
  const uint32_t bar0 = stg0 + DZI_EPI_WARPS * DZI_STG_BYTES;
  const uint32_t full0 = bar0;
  const uint32_t empty0 = bar0 + 8u * STAGES;
  const uint32_t tfull0 = bar0 + 16u * STAGES;
  const uint32_t tempty0 = tfull0 + 16u;
  const uint32_t done_bar = tempty0 + 16u;
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
      mbar_init(tempty0 + 8u * b, 2 * DZI_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch(&map_h);
    tma_prefetch(&map_w);
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
  const uint32_t peer_empty0 = mapa_shared(empty0, 1);
  const uint32_t peer_tfull0 = mapa_shared(tfull0, 1);

  if (warp == 0 || warp >= DZI_PW) {
    // ------------------------------------------------------------ TMA producers (both CTAs, whole warp)
    // stage s belongs to producer s % DZI_PROD
    const int prod = warp == 0 ? 0 : warp - DZI_PW + 1;
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int rt, uv, vt0, vt1;
      dzi_unit(a, u, rt, uv, vt0, vt1);
      const int row0 = rt * DZI_ROWS + (int)rank * (DZI_ROWS / 2);
      for (int vt = vt0; ok && vt < vt1; ++vt) {
        const int wrow = a.v_begin + vt * DZI_BN + (int)rank * (DZI_BN / 2);
        for (int kb = 0; kb < a.n_kb; ++kb) {
          if (stage % DZI_PROD == prod) {
            if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
            if (elect_one()) {
              const uint32_t sa = sbase + stage * DZI_STAGE_BYTES;
              const uint32_t fb = lead_full0 + 8u * stage;
              if (leader) mbar_arrive_expect_tx(full0 + 8u * stage, 2 * DZI_STAGE_BYTES);
              if (G8) tma_load_4d_pair(sa, &map_h, fb, kb * BK, 0, 0, row0 / 8);
              else tma_load_3d_pair(sa, &map_h, fb, kb * BK, 0, row0);
              tma_load_2d_pair(sa + DZI_A_BYTES, &map_w, fb, kb * BK, wrow);
              if (!leader) mbar_arrive_cluster(fb);
            }
            __syncwarp();
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    if (leader && prod == 0) drain_loads<STAGES>(full0, stage, phase, issued);
  } else if (warp == 1) {
    if (leader) {
      // ------------------------------------------------------------ pair MMA issuer (leader, whole warp)
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, DZI_BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      bool ok = true;
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int rt, uv, vt0, vt1;
        dzi_unit(a, u, rt, uv, vt0, vt1);
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          if (!warp_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + buf * DZI_BN;
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!warp_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
            tc_fence_after();
            if (elect_one()) {
              const uint32_t sa = sbase + stage * DZI_STAGE_BYTES;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_bf16_pair(d, desc_kmajor(sa, k), desc_kmajor(sa + DZI_A_BYTES, k), idesc, (kb | k) != 0);
              mma_commit_pair(empty0 + 8u * stage);
              mma_commit_pair(peer_empty0 + 8u * stage);
            }
            __syncwarp();
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
          if (ok && elect_one()) {
            mma_commit_pair(tfull0 + 8u * buf);
            mma_commit_pair(peer_tfull0 + 8u * buf);
          }
          __syncwarp();
        }
      }
      if (elect_one()) mma_commit_pair(done_bar);
      __syncwarp();
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int hf = (warp - EPI_WARP0) >> 2;   // 128-column half of the tile
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(hf * (DZI_BN / 2));
    const uint32_t stg = stg0 + (uint32_t)(warp - EPI_WARP0) * DZI_STG_BYTES;
    const uint64_t pol = l2_evict_first_policy();   // dZ is streamed out once, read by the next kernel
    const float sl2f = a.scale_log2;
    int tcount = 0;
    int sbuf = 0;
    bool ok = true;
    if (MODE == MODE_STATS) {
      // thread (t4, tq): token rows y0 + t4 and y0 + 8 + t4, columns 8k + 2 tq + {0, 1} of each 32
      const int t4 = lane >> 2, tq = lane & 3;
      const uint64_t sl2 = f2_pack(sl2f, sl2f);
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int rt, uv, vt0, vt1;
        dzi_unit(a, u, rt, uv, vt0, vt1);
        const int y0 = rt * DZI_ROWS + (int)rank * (DZI_ROWS / 2) + q * 16;
        float sa[5] = {NEG_BIG, 0.f, NEG_BIG, 0.f, 0.f}, sb[5] = {NEG_BIG, 0.f, NEG_BIG, 0.f, 0.f};
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          if (!warp_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tbase = lane_addr + buf * DZI_BN;
#pragma unroll 1
          for (int c = 0; c < (DZI_BN / 2) / 32; ++c) {
            const int x = vt * DZI_BN + hf * (DZI_BN / 2) + c * 32;   // first column of this chunk
            if (x >= a.v_count) break;                               // warp-uniform
            uint32_t ra[16], rb[16];
            tmem_ld16x256b_x4(tbase + c * 32, ra);
            tmem_ld16x256b_x4(tbase + c * 32 + (16u << 16), rb);
            tmem_wait_ld16(ra, rb);
            const int col0 = x + 2 * tq;
            if (x + 32 <= a.v_count) {
              dzi_g8_stats<SV, false>(ra, sl2, col0, a.v_count, sa);
              dzi_g8_stats<SV, false>(rb, sl2, col0, a.v_count, sb);
            } else {
              dzi_g8_stats<SV, true>(ra, sl2, col0, a.v_count, sa);
              dzi_g8_stats<SV, true>(rb, sl2, col0, a.v_count, sb);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader) mbar_arrive(tempty0 + 8u * buf);
            else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
          }
        }
        dzi_stats_merge(sa, 1);
        dzi_stats_merge(sb, 1);
        dzi_stats_merge(sa, 2);
        dzi_stats_merge(sb, 2);
        if (ok && tq == 0) {
          float* pr = a.partials + (size_t)(uv * DZI_CSPLIT + hf) * 5 * a.n_rows;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int row = y0 + 8 * h2 + t4;
            const float* v = h2 ? sb : sa;
            if (row < a.n_rows)
              for (int i = 0; i < 5; ++i) pr[(size_t)i * a.n_rows + row] = v[i];
          }
        }
      }
    } else if (G8) {
      // thread (t4, tq) = (lane / 4, lane % 4): token rows y0 + t4 (16-lane group 0) and y0 + 8 + t4
      // (group 1), columns 8k + 2 tq + {0, 1} of each 32; staging rows t4 and 8 + t4
      const int t4 = lane >> 2, tq = lane & 3;
      const uint64_t sl2 = f2_pack(sl2f, sl2f);
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int rt, uv, vt0, vt1;
        dzi_unit(a, u, rt, uv, vt0, vt1);
        const int y0 = rt * DZI_ROWS + (int)rank * (DZI_ROWS / 2) + q * 16;   // first token row of this warp
        const DziRow rA = dzi_row(a, y0 + t4), rB = dzi_row(a, y0 + 8 + t4);
        const bool anyA = __any_sync(0xffffffffu, rA.live), anyB = __any_sync(0xffffffffu, rB.live);
        const uint64_t nlsA = f2_pack(-rA.Ls, -rA.Ls), nltA = f2_pack(-rA.Lt, -rA.Lt);
        const uint64_t nlsB = f2_pack(-rB.Ls, -rB.Ls), nltB = f2_pack(-rB.Lt, -rB.Lt);
        const uint64_t cfA = f2_pack(rA.coef, rA.coef), cfB = f2_pack(rB.coef, rB.coef);
        uint64_t accA = 0, accB = 0;   // packed (0.f, 0.f)
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          if (!warp_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tbase = lane_addr + buf * DZI_BN;
#pragma unroll 1
          for (int cp = 0; cp < (DZI_BN / 2) / DZI_STORE_COLS; ++cp) {
            const int x0 = vt * DZI_BN + hf * (DZI_BN / 2) + cp * DZI_STORE_COLS;   // chunk-relative column
            if (x0 >= a.v_count) break;                                            // warp-uniform
            // the staging buffer is free once the store issued from it two blocks ago has read it
            if (lane == 0) bulk_wait_read1();
            __syncwarp();
            const uint32_t sb = stg + (uint32_t)sbuf * 2048u;
#pragma unroll
            for (int c = 0; c < DZI_STORE_COLS / 32; ++c) {
              const uint32_t col = tbase + cp * DZI_STORE_COLS + c * 32;
              uint32_t ra[16], rb[16];
              if (anyA) tmem_ld16x256b_x4(col, ra);
              if (anyB) tmem_ld16x256b_x4(col + (16u << 16), rb);
              if (anyA && anyB) tmem_wait_ld16(ra, rb);
              else if (anyA) tmem_wait_ld16(ra);
              else if (anyB) tmem_wait_ld16(rb);
              const int col0 = x0 + c * 32 + 2 * tq;     // column of r[0] (chunk-relative)
              const bool full = x0 + c * 32 + 32 <= a.v_count;
              uint32_t pa[4] = {0u, 0u, 0u, 0u}, pb[4] = {0u, 0u, 0u, 0u};
              if (anyA) {
                if (full) dzi_g8_chunk<SV, false>(ra, sl2, nlsA, nltA, cfA, col0, a.v_count, pa, accA);
                else dzi_g8_chunk<SV, true>(ra, sl2, nlsA, nltA, cfA, col0, a.v_count, pa, accA);
              }
              if (anyB) {
                if (full) dzi_g8_chunk<SV, false>(rb, sl2, nlsB, nltB, cfB, col0, a.v_count, pb, accB);
                else dzi_g8_chunk<SV, true>(rb, sl2, nlsB, nltB, cfB, col0, a.v_count, pb, accB);
              }
              // 16-byte chunk j of 128-byte staging row rr sits at j ^ (rr % 8); rows t4 and 8 + t4
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t off = ((((uint32_t)(4 * c + k)) ^ (uint32_t)t4) << 4) + 4u * tq;
                st_shared_b32(sb + (uint32_t)t4 * 128u + off, pa[k]);
                st_shared_b32(sb + (uint32_t)(8 + t4) * 128u + off, pb[k]);
              }
            }
            fence_async_shared();
            __syncwarp();
            if (lane == 0) {
              if (y0 < a.n_rows) tma_store_2d_hint(&map_out, sb, x0, y0, pol);
              bulk_commit();
            }
            sbuf ^= 1;
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader) mbar_arrive(tempty0 + 8u * buf);
            else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
          }
        }
        // cross term of each row: the four threads of a row (tq = 0..3) and both packed lanes
        float a0, a1, b0, b1;
        f2_unpack(accA, a0, a1);
        f2_unpack(accB, b0, b1);
        float xa = a0 + a1, xb = b0 + b1;
        xa += __shfl_xor_sync(0xffffffffu, xa, 1);
        xb += __shfl_xor_sync(0xffffffffu, xb, 1);
        xa += __shfl_xor_sync(0xffffffffu, xa, 2);
        xb += __shfl_xor_sync(0xffffffffu, xb, 2);
        if (ok && tq == 0 && a.a_parts) {
          float* ap = a.a_parts + (size_t)(a.a_part_base + uv * DZI_CSPLIT + hf) * a.n_rows;
          if (y0 + t4 < a.n_rows) ap[y0 + t4] = xa * sl2f;
          if (y0 + 8 + t4 < a.n_rows) ap[y0 + 8 + t4] = xb * sl2f;
        }
      }
    } else {
      const bool odd = (lane & 1) != 0;               // odd lanes take columns 16..31 of a chunk
      const bool mine_s = (int)(lane & 1) == a.s_view;
      const int sub = lane >> 1;                      // token row within the warp's 16
      // 16-byte chunk k of 128-byte staging row r sits at chunk k ^ (r % 8) (128-byte swizzle)
      const uint32_t rowoff = (uint32_t)sub * 128u;
      const uint32_t swz = (uint32_t)(sub & 7);
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int rt, uv, vt0, vt1;
        dzi_unit(a, u, rt, uv, vt0, vt1);
        const int y0 = rt * DZI_ROWS + (int)rank * (DZI_ROWS / 2) + q * 16;   // first token row of this warp
        const int row = y0 + sub;
        const DziRow rr = dzi_row(a, row);
        const bool any = __any_sync(0xffffffffu, rr.live);
        // e = 2^(u - L) of this lane's view ("me") and of the partner's ("ot"); dZ = coef (q - p)
        const float L_me = mine_s ? rr.Ls : rr.Lt, L_ot = mine_s ? rr.Lt : rr.Ls;
        const float c_me = mine_s ? rr.coef : -rr.coef;
        float acc_me = 0.f, acc_ot = 0.f;   // sum e (z_me - z_ot) over valid columns, per view
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          // warp-uniform outcome: the lanes exchange values by shuffles below
          if (!warp_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tbase = lane_addr + buf * DZI_BN;
#pragma unroll 1
          for (int cp = 0; cp < (DZI_BN / 2) / DZI_STORE_COLS; ++cp) {
            const int x0 = vt * DZI_BN + hf * (DZI_BN / 2) + cp * DZI_STORE_COLS;   // chunk-relative column
            if (x0 >= a.v_count) break;                                            // warp-uniform
            if (lane == 0) bulk_wait_read1();
            __syncwarp();
            const uint32_t sb = stg + (uint32_t)sbuf * 2048u + rowoff;
#pragma unroll
            for (int c = 0; c < DZI_STORE_COLS / 32; ++c) {
              uint32_t pk[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
              if (any) {
                uint32_t v[32];
                tmem_ld32_raw(tbase + cp * DZI_STORE_COLS + c * 32, v);
                tmem_wait_ld_regs(v);
                const int nvalid = a.v_count - (x0 + c * 32) - (odd ? 16 : 0);
                float me[16], ot[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const float lo = __uint_as_float(v[j]), hi = __uint_as_float(v[16 + j]);
                  ot[j] = __shfl_xor_sync(0xffffffffu, odd ? lo : hi, 1);
                  me[j] = odd ? hi : lo;
                }
                float am0 = 0.f, am1 = 0.f, ao0 = 0.f, ao1 = 0.f;
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                  const float em0 = ex2(fmaf(me[j], sl2f, -L_me)), em1 = ex2(fmaf(me[j + 1], sl2f, -L_me));
                  const float eo0 = ex2(fmaf(ot[j], sl2f, -L_ot)), eo1 = ex2(fmaf(ot[j + 1], sl2f, -L_ot));
                  pk[j / 2] = pack_bf16x2(c_me * (em0 - eo0), c_me * (em1 - eo1));
                  const float d0 = me[j] - ot[j], d1 = me[j + 1] - ot[j + 1];
                  const bool v0 = j < nvalid, v1 = j + 1 < nvalid;
                  am0 = fmaf(v0 ? em0 : 0.f, d0, am0);
                  am1 = fmaf(v1 ? em1 : 0.f, d1, am1);
                  ao0 = fmaf(v0 ? eo0 : 0.f, d0, ao0);
                  ao1 = fmaf(v1 ? eo1 : 0.f, d1, ao1);
                }
                acc_me += am0 + am1;
                acc_ot += ao0 + ao1;
              }
              // this thread's 16 columns = 16-byte chunks k0, k0 + 1 of its staging row
              const uint32_t k0 = (uint32_t)(c * 4 + (odd ? 2 : 0));
              st_shared_v4(sb + ((k0 ^ swz) << 4), pk[0], pk[1], pk[2], pk[3]);
              st_shared_v4(sb + (((k0 + 1) ^ swz) << 4), pk[4], pk[5], pk[6], pk[7]);
            }
            fence_async_shared();
            __syncwarp();
            if (lane == 0) {
              if (y0 < a.n_rows) tma_store_2d_hint(&map_out, stg + (uint32_t)sbuf * 2048u, x0, y0, pol);
              bulk_commit();
            }
            sbuf ^= 1;
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader) mbar_arrive(tempty0 + 8u * buf);
            else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
          }
        }
        // cross term p (z_t - z_s) = e_t (z_t - z_s): the student lane holds -acc_ot, the teacher lane acc_me
        const float part = mine_s ? -acc_ot : acc_me;
        const float cross = part + __shfl_xor_sync(0xffffffffu, part, 1);
        if (ok && row < a.n_rows && !odd && a.a_parts)
          a.a_parts[(size_t)(a.a_part_base + uv * DZI_CSPLIT + hf) * a.n_rows + row] = cross * sl2f;
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
