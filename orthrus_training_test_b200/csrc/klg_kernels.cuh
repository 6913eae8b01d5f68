// sm_100a kernels of the fused KL-GEMM distillation loss.
//
// Notation: N rows (student/teacher pairs), H hidden, V vocab, W = lm_head [V, H].
// Logits are z = h W^T / T.  All softmax arithmetic runs in the log2 domain:
// u = z * log2(e) / T, so exp(z - m) = 2^(u - m2).
//
//  lse_pair_kernel     training pass 1: per view, online (max, sum 2^(u - max)) per row
//                      over all vocab tiles (row block resident for H <= 576).
//  dual_pair_kernel    both views' logit tiles per (row pair tile, vocab tile), one MMA per
//                      view (the row-major form; the interleaved-view kernel of
//                      klg_dzi.cuh, one MMA for both views, is the default for both modes):
//     <MODE_DZ>        training pass 2: dZ = g valid/count (q - p)/T as bf16 for one vocab
//                      chunk, plus the KL cross term sum_v p (u_t - u_s) per unit (the
//                      fp32-faithful path's two dZ planes; bf16 with KLG_DZI=0);
//     <MODE_STATS>     forward only: per unit the online (m_s, S_s, m_t, S_t, A) record
//                      (N % 8 != 0 or KLG_DZI=0).
//  gemm_pair_kernel    C (+)= A B over one backward chunk: dW_chunk = dZ^T h_s and
//                      dH += dZ W_chunk in one launch (host-built longest-first schedule).
//
// All three run on CTA pairs (cluster of 2, tcgen05.mma.cta_group::2, M = 256).  Warp
// roles: warp 0 (+ extra producer warps after the epilogue) issue TMA loads, warp 1
// allocates TMEM and issues the MMAs, the other warps are the epilogue (warp w reads TMEM
// lane quarter w % 4: one output row per thread).  Shared-memory stages are recycled
// through full/empty mbarriers, the two TMEM accumulator buffers through tmem_full /
// tmem_empty so the epilogue of tile j overlaps the MMAs of tile j+1.
#pragma once
#include "klg_ptx.cuh"

namespace klg {

constexpr int BM = 128;                     // rows per tile (TMEM lanes)
constexpr int BK = 64;                      // bf16 elements per k-block (one 128 B swizzle row)
constexpr int TILE_128x64 = BM * BK * 2;    // 16 KB
constexpr int EPI_WARP0 = 2;                // warp 0: TMA producer, warp 1: MMA issuer, then epilogue warps
constexpr float NEG_BIG = -1.0e30f;

// =====================================================================================
// per-(row pair tile, vocab range) work units shared by the dual-view kernels
// =====================================================================================
constexpr int DUAL_TMEM_COLS = 512;                // 2 buffers x (Z_s 128 | Z_t 128)

struct DualArgs {
  int n_rows;       // N
  int v_begin;      // first W row of this launch
  int v_count;      // W rows covered by this launch
  int n_rt;         // ceil(N / 256): 256-row pair tiles
  int n_vt;         // ceil(v_count / 128)
  int vt_per_unit;  // vocab tiles per work unit
  int n_units;      // n_rt * ceil(n_vt / vt_per_unit)
  int n_kb;         // ceil(H / 64)
  float scale_log2; // log2(e) / T
  // MODE_STATS
  float* partials;  // [n_uv * DZP_CSPLIT][5][N]
  // MODE_DZ
  const float* lse;      // [2][N] log2-domain log-sum-exp (student, teacher)
  const uint8_t* mask;   // [N]
  const float* count;    // device scalar: number of valid rows (global)
  const float* grad;     // device scalar: upstream gradient, or nullptr for 1
  float inv_temp;
  __nv_bfloat16* dz;     // [N][ld_dz], column j = W row v_begin + j
  int ld_dz;
  float* a_parts;        // optional [.][N]: per unit sum_v p_v (u_t - u_s) (log2 units), row a_part_base + uv
  int a_part_base;
};

// Units are numbered row-tile-major: the pairs that run at the same time share a few row
// tiles (both views: 2 x 256 rows x H), so the rows stay in L2 while each pair sweeps its own
// vocabulary range.  (Numbered vocab-range-major, 74 pairs stream 74 different row tiles:
// 148 MB at H = 2048, more than L2, and every vocabulary tile re-reads its rows from DRAM.)
__device__ __forceinline__ void dual_unit(const DualArgs& a, int u, int& rt, int& uv, int& vt0, int& vt1) {
  const int n_uv = (a.n_vt + a.vt_per_unit - 1) / a.vt_per_unit;
  rt = u / n_uv;
  uv = u - rt * n_uv;
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

// One 32-column chunk of the pass-1 statistics update (online max / sum-exp / KL).
__device__ __forceinline__ void stats_chunk(const uint32_t (&bs)[32], const uint32_t (&bt)[32], int nvalid, float sl2,
                                            float& ms, float& Ss, float& mt, float& St, float& A) {
  float zs[32], zt[32];
  float cms = -INFINITY, cmt = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const bool v = j < nvalid;
    zs[j] = v ? __uint_as_float(bs[j]) * sl2 : -INFINITY;
    zt[j] = v ? __uint_as_float(bt[j]) * sl2 : -INFINITY;
    cms = fmaxf(cms, zs[j]);
    cmt = fmaxf(cmt, zt[j]);
  }
  const float nms = fmaxf(ms, cms);
  const float nmt = fmaxf(mt, cmt);
  const float rs = ex2(ms - nms);
  const float rt = ex2(mt - nmt);
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
  St = fmaf(St, rt, t0 + t1);
  A = fmaf(A, rt, a0 + a1);
}

// One 32-column chunk of dZ = coef * (2^(u_s - L_s) - 2^(u_t - L_t)) as 16 bf16 pairs,
// and acc += sum_{j < nvalid} p_j (z_t - z_s) (raw logits; scaled by log2(e)/T later).
// Rows outside the loss (live = false: mask off, or no valid row at all) get zeros.
__device__ __forceinline__ void dz_chunk(const uint32_t (&bs)[32], const uint32_t (&bt)[32], int nvalid, float sl2,
                                         float Ls, float Lt, float coef, bool live, uint32_t (&pk)[16], float& acc) {
  if (!live) {
#pragma unroll
    for (int j = 0; j < 16; ++j) pk[j] = 0u;
    return;
  }
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float zs0 = __uint_as_float(bs[j]), zs1 = __uint_as_float(bs[j + 1]);
    const float zt0 = __uint_as_float(bt[j]), zt1 = __uint_as_float(bt[j + 1]);
    const float q0 = ex2(fmaf(zs0, sl2, -Ls));
    const float q1 = ex2(fmaf(zs1, sl2, -Ls));
    const float p0 = ex2(fmaf(zt0, sl2, -Lt));
    const float p1 = ex2(fmaf(zt1, sl2, -Lt));
    pk[j / 2] = pack_bf16x2(coef * (q0 - p0), coef * (q1 - p1));
    a0 = fmaf(j < nvalid ? p0 : 0.f, zt0 - zs0, a0);
    a1 = fmaf(j + 1 < nvalid ? p1 : 0.f, zt1 - zs1, a1);
  }
  acc += a0 + a1;
}

// dz_chunk for the fp32-faithful path: dZ as two bf16 planes, hi = bf16(d) and
// lo = bf16(d - hi), so hi + lo carries d to ~2^-16 relative.
__device__ __forceinline__ void dz_chunk_split(const uint32_t (&bs)[32], const uint32_t (&bt)[32], int nvalid,
                                               float sl2, float Ls, float Lt, float coef, uint32_t (&ph)[16],
                                               uint32_t (&pl)[16], float& acc) {
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float zs0 = __uint_as_float(bs[j]), zs1 = __uint_as_float(bs[j + 1]);
    const float zt0 = __uint_as_float(bt[j]), zt1 = __uint_as_float(bt[j + 1]);
    const float q0 = ex2(fmaf(zs0, sl2, -Ls));
    const float q1 = ex2(fmaf(zs1, sl2, -Ls));
    const float p0 = ex2(fmaf(zt0, sl2, -Lt));
    const float p1 = ex2(fmaf(zt1, sl2, -Lt));
    const float d0 = coef * (q0 - p0), d1 = coef * (q1 - p1);
    const __nv_bfloat162 h = __floats2bfloat162_rn(d0, d1);
    ph[j / 2] = *reinterpret_cast<const uint32_t*>(&h);
    pl[j / 2] = pack_bf16x2(d0 - __low2float(h), d1 - __high2float(h));
    a0 = fmaf(j < nvalid ? p0 : 0.f, zt0 - zs0, a0);
    a1 = fmaf(j + 1 < nvalid ? p1 : 0.f, zt1 - zs1, a1);
  }
  acc += a0 + a1;
}

// =====================================================================================
// pass-1 log-sum-exp on CTA pairs (training path)
//
// One view at a time (student rows, then teacher rows): per unit (view, 256-row pair
// tile, vocab range) the pair computes 256 x 256 logit tiles with
// tcgen05.mma.cta_group::2 (each CTA: its own 128 rows as A, its half of the W tile as
// B) into double-buffered TMEM, and LSE_CSPLIT epilogue warps per TMEM lane quarter
// (each owning a column slice of the tile) keep online (m, S) per row.  Output: partial
// records parts[n_uv * LSE_CSPLIT][2][2N] = (m, S) in log2 units, row index view*N + row.
// The KL cross term is accumulated by the dZ pass, which has both views' values.
// =====================================================================================
constexpr int LSE_BN = 256;                                // vocab rows per pair tile
#ifndef KLG_LSE_STAGES
#define KLG_LSE_STAGES 6
#endif
constexpr int LSE_STAGES = KLG_LSE_STAGES;
constexpr int LSE_A_BYTES = TILE_128x64;                   // this CTA's 128 rows x 64
constexpr int LSE_B_BYTES = (LSE_BN / 2) * BK * 2;         // this CTA's half of the W tile
constexpr int LSE_STAGE_BYTES = LSE_A_BYTES + LSE_B_BYTES; // 32 KB
#ifndef KLG_EPI_SPLIT
#define KLG_EPI_SPLIT 2
#endif
constexpr int LSE_CSPLIT = KLG_EPI_SPLIT;                  // epilogue warps per TMEM lane quarter
constexpr int LSE_EPI_WARPS = 4 * LSE_CSPLIT;
constexpr int LSE_COLS_PER_WARP = LSE_BN / LSE_CSPLIT;
#ifndef KLG_LSE_PROD
#define KLG_LSE_PROD 2
#endif
constexpr int LSE_PROD = KLG_LSE_PROD;                      // producer warps (round-robin load steps)
constexpr int LSE_PW = EPI_WARP0 + LSE_EPI_WARPS;           // first extra producer warp
constexpr int LSE_THREADS = 32 * (LSE_PW + LSE_PROD - 1);
constexpr int LSE_TMEM_COLS = 512;                         // 2 buffers x 256 columns
constexpr int LSE_SMEM = 1024 + LSE_STAGES * LSE_STAGE_BYTES + 256;
// Resident-A variant (H <= 576): the CTA's 128 x H row block stays in shared memory for a
// whole unit and only the W halves stream, halving the bytes TMA writes per MMA.
constexpr int LSE_RES_MAX_KB = 9;
#ifndef KLG_LSE_RES_STAGES
#define KLG_LSE_RES_STAGES 4   // 5 fits but measured no faster
#endif
constexpr int LSE_RES_STAGES = KLG_LSE_RES_STAGES;
constexpr int LSE_RES_SMEM = 1024 + LSE_RES_MAX_KB * LSE_A_BYTES + LSE_RES_STAGES * LSE_B_BYTES + 256;

struct LseArgs {
  int n_rows;       // N rows per view
  int vocab;        // V
  int n_rp;         // ceil(N / 256)
  int n_vt;         // ceil(V / 256)
  int vt_per_unit;
  int n_uv;         // ceil(n_vt / vt_per_unit)
  int n_units;      // 2 * n_rp * n_uv
  int n_kb;         // ceil(H / 64)
  float scale_log2; // log2(e) / T
  float* parts;     // EPI_LSE: [n_uv * LSE_CSPLIT][2][n_views * N]; else [n_uv * rep * LSE_CSPLIT][5][N]
  int n_views;      // 2: student rows then teacher rows (training pass 1); 1: one matrix (EPI_SAMPLE)
  uint32_t seed_lo, seed_hi;   // EPI_SAMPLE
  // Filtered sampling (top-k / top-p): EPI_GREEDY also writes each row's 32-column chunk
  // maxima cmax[row][n_ck] (raw logits) when cmax is set; EPI_CAND appends every logit
  // z >= thr[row] with its column to the row's candidate list (cand_z / cand_i [row][cap],
  // counter cand_cnt[row]; entries past cap are counted, not stored).
  float* cmax;
  int n_ck;
  const float* thr;
  int* cand_cnt;
  float* cand_z;
  int* cand_i;
  int cap;
  // Row replication (EPI_GREEDY / EPI_SAMPLE with N <= 128, one row tile): the pair tile's
  // 256 M rows hold `rep` copies of rows 0..256/rep-1, and the copy j of a warp's rows
  // takes the j-th 1/rep of the tile's columns -- every epilogue warp gets work instead of
  // the few whose TMEM lanes hold the real rows.  rep = 1: none; 2: each CTA loads rows
  // 0..127 with map_hs; 4: each CTA loads rows 0..63 twice with map_ht (box 64 rows).
  int rep;
};

// EPI_LSE: (m, S) per row and view (training pass 1).  EPI_GREEDY: (m, S) and the argmax of
// z.  EPI_SAMPLE: (m, S) and a Gumbel-max draw from softmax(z / T).
enum { EPI_LSE = 0, EPI_GREEDY = 1, EPI_SAMPLE = 2, EPI_CAND = 3 };
constexpr uint32_t HASH_ROW = 0x9E3779B1u, HASH_COL = 0x85EBCA77u, HASH_SEED = 0xC2B2AE3Du;

// Counter-based 32-bit hash of (seed, row, column): the three keys combined with odd
// multipliers, then the "lowbias32" avalanche finaliser (public domain).  The oracle
// restates it bit for bit.
__host__ __device__ __forceinline__ uint32_t hash_mix(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return x;
}

__host__ __device__ __forceinline__ uint32_t sample_hash(uint32_t seed_lo, uint32_t seed_hi, uint32_t row, uint32_t col) {
  return hash_mix(seed_lo ^ (row * HASH_ROW) ^ (col * HASH_COL) ^ (seed_hi * HASH_SEED));
}

__device__ __forceinline__ void lse_unit(const LseArgs& a, int u, int& view, int& rp, int& uv, int& vt0, int& vt1) {
  const int per_uv = a.n_views * a.n_rp;
  uv = u / per_uv;
  const int r = u % per_uv;
  view = r / a.n_rp;
  rp = r % a.n_rp;
  vt0 = uv * a.vt_per_unit;
  vt1 = min(vt0 + a.vt_per_unit, a.n_vt);
}

// Online (m, S) update of one 32-column chunk, log2 units.
__device__ __forceinline__ void lse_chunk(const uint32_t (&b)[32], int nvalid, float sl2, float& m, float& S) {
  float cm = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) cm = fmaxf(cm, j < nvalid ? __uint_as_float(b[j]) : -INFINITY);
  const float nm = fmaxf(m, cm * sl2);
  const float r = ex2(m - nm);
  m = nm;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    s0 += j < nvalid ? ex2(fmaf(__uint_as_float(b[j]), sl2, -m)) : 0.f;
    s1 += j + 1 < nvalid ? ex2(fmaf(__uint_as_float(b[j + 1]), sl2, -m)) : 0.f;
    s2 += j + 2 < nvalid ? ex2(fmaf(__uint_as_float(b[j + 2]), sl2, -m)) : 0.f;
    s3 += j + 3 < nvalid ? ex2(fmaf(__uint_as_float(b[j + 3]), sl2, -m)) : 0.f;
  }
  S = fmaf(S, r, (s0 + s1) + (s2 + s3));
}

// Exponential variate in log2 units, E = -log2(1 - V), from the hash's top 23 bits:
// V = (2k + 1) 2^-24 in [2^-24, 1 - 2^-24], exact in fp32 (the float 1.k minus 1 - 2^-24).
// Small V (the large-key tail of the Gumbel variate) takes the series of -ln(1 - V), whose
// truncation error is below 2^-32 relative for V < 1/32; elsewhere 1 - V >= 31/32 and
// lg2.approx carries ~2^-22 absolute error on a result >= 0.045.
__device__ __forceinline__ float uniform_open(uint32_t x) {
  return __uint_as_float(0x3F800000u | (x >> 9)) - 0.99999994039535522461f;
}

__device__ __forceinline__ float exp_variate_log2(uint32_t x) {
  const float v = uniform_open(x);
  const float ser = v * fmaf(v, fmaf(v, fmaf(v, fmaf(v, fmaf(v, 1.f / 6.f, 0.2f), 0.25f), 1.f / 3.f), 0.5f), 1.f) *
                    1.44269504088896341f;
  return v < 0.03125f ? ser : -__log2f(1.f - v);
}

// Online (m, S) and best-key update of one 32-column chunk (columns col0..col0+31 of this
// thread's row), branch-free, with trees instead of serial chains.  Greedy keys are the raw
// logits; sampling keys are u - log2(E), u = z log2(e) / T and E the exponential variate of
// (seed, row, column) -- the Gumbel-max rule (the argmax of u + Gumbel noise is a draw from
// softmax(z / T)) with the constant log2(ln 2) dropped.  Ties keep the lowest column: the
// tree takes the right (higher) operand only when strictly greater, and a chunk replaces
// the running best (from lower columns) only when strictly greater.
// rk = seed_lo ^ row * HASH_ROW ^ seed_hi * HASH_SEED, so rk ^ col * HASH_COL is sample_hash's key.
template <bool SAMPLE>
__device__ __forceinline__ void select_chunk(const uint32_t (&b)[32], int nvalid, int col0, float sl2, uint32_t rk,
                                             float& m, float& S, float& bk, int& bi, float& bz, float& cmx) {
  float z[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) z[j] = j < nvalid ? __uint_as_float(b[j]) : -INFINITY;
  float t[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) t[j] = fmaxf(z[2 * j], z[2 * j + 1]);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) t[j] = fmaxf(t[2 * j], t[2 * j + 1]);
  cmx = t[0];
  const float nm = fmaxf(m, t[0] * sl2);
  const float r = ex2(m - nm);
  m = nm;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;   // ex2(-inf) = 0 for the invalid columns
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    s0 += ex2(fmaf(z[j], sl2, -m));
    s1 += ex2(fmaf(z[j + 1], sl2, -m));
    s2 += ex2(fmaf(z[j + 2], sl2, -m));
    s3 += ex2(fmaf(z[j + 3], sl2, -m));
  }
  S = fmaf(S, r, (s0 + s1) + (s2 + s3));

  float k[32];
  if (SAMPLE) {
    const uint32_t cb = (uint32_t)col0 * HASH_COL;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const uint32_t x = hash_mix(rk ^ (cb + (uint32_t)j * HASH_COL));
      k[j] = fmaf(z[j], sl2, -__log2f(exp_variate_log2(x)));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) k[j] = z[j];
  }
  float kk[16], zz[16];
  int ii[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const bool right = k[2 * j + 1] > k[2 * j];
    kk[j] = right ? k[2 * j + 1] : k[2 * j];
    ii[j] = 2 * j + (right ? 1 : 0);
    if (SAMPLE) zz[j] = right ? z[2 * j + 1] : z[2 * j];
  }
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) {
      const bool right = kk[2 * j + 1] > kk[2 * j];
      kk[j] = right ? kk[2 * j + 1] : kk[2 * j];
      ii[j] = right ? ii[2 * j + 1] : ii[2 * j];
      if (SAMPLE) zz[j] = right ? zz[2 * j + 1] : zz[2 * j];
    }
  const bool take = kk[0] > bk;
  bk = take ? kk[0] : bk;
  bi = take ? col0 + ii[0] : bi;
  bz = take ? (SAMPLE ? zz[0] : kk[0]) : bz;
}

template <bool RES, int EPI>
__global__ void __launch_bounds__(LSE_THREADS, 1)
lse_pair_kernel(const __grid_constant__ CUtensorMap map_hs, const __grid_constant__ CUtensorMap map_ht,
                const __grid_constant__ CUtensorMap map_w, const LseArgs a) {
  constexpr int STAGES = RES ? LSE_RES_STAGES : LSE_STAGES;
  constexpr int NPROD = LSE_PROD;
  constexpr int STAGE_BYTES = RES ? LSE_B_BYTES : LSE_STAGE_BYTES;   // W half [+ A k-block]
  constexpr int A_REGION = RES ? LSE_RES_MAX_KB * LSE_A_BYTES : 0;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t abase = smem_u32(smem);               // resident A (RES)
  const uint32_t sbase = abase + A_REGION;             // stage ring
  const uint32_t bar0 = sbase + STAGES * STAGE_BYTES;
  const uint32_t full0 = bar0;                         // [STAGES] leader only: both CTAs' bytes
  const uint32_t empty0 = bar0 + 8u * STAGES;          // [STAGES] each CTA
  const uint32_t tfull0 = bar0 + 16u * STAGES;         // [2] each CTA
  const uint32_t tempty0 = tfull0 + 16u;               // [2] leader only: warp arrivals of both CTAs
  const uint32_t done_bar = tempty0 + 16u;
  const uint32_t afull_bar = done_bar + 8u;            // RES: leader only, both CTAs' A bytes
  const uint32_t aempty_bar = afull_bar + 8u;          // RES: each CTA
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
      mbar_init(tempty0 + 8u * b, 2 * LSE_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    mbar_init(afull_bar, 2);
    mbar_init(aempty_bar, 1);
    fence_mbar_init();
    tma_prefetch(&map_hs);
    tma_prefetch(&map_ht);
    tma_prefetch(&map_w);
  }
  if (warp == 1) tmem_alloc_pair(smem_u32(&tmem_slot), LSE_TMEM_COLS);
  tc_fence_before();
  cluster_sync();   // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_enter();   // inputs of this launch are complete from here on
  volatile int* abort_p = &abort_flag;
  const uint32_t lead_full0 = mapa_shared(full0, 0);
  const uint32_t lead_tempty0 = mapa_shared(tempty0, 0);
  const uint32_t lead_afull = mapa_shared(afull_bar, 0);
  const uint32_t peer_empty0 = mapa_shared(empty0, 1);
  const uint32_t peer_tfull0 = mapa_shared(tfull0, 1);
  const uint32_t peer_aempty = mapa_shared(aempty_bar, 1);

  if (warp == 0 || warp >= LSE_PW) {
    // producer warps: warp 0 and warps LSE_PW.. take the pipeline's load steps round-robin
    const int prod = warp == 0 ? 0 : warp - LSE_PW + 1;
    {
      // ------------------------------------------------------------ TMA producer (both CTAs, whole warp)
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      int ucount = 0;
      bool ok = true;
      for (int u = cid; ok && u < a.n_units; u += n_clusters, ++ucount) {
        int view, rp, uv, vt0, vt1;
        lse_unit(a, u, view, rp, uv, vt0, vt1);
        const CUtensorMap* ma = view ? &map_ht : &map_hs;
        const int row0 = rp * 256 + (int)rank * 128;
        // this CTA's 128 A rows of k-block kb (replicated rows when a.rep > 1)
        auto load_a = [&](uint32_t dst, uint32_t bar, int kb) {
          if (a.rep == 1) {
            tma_load_2d_pair(dst, ma, bar, kb * BK, row0);
          } else if (a.rep == 2) {
            tma_load_2d_pair(dst, &map_hs, bar, kb * BK, 0);
          } else {
            tma_load_2d_pair(dst, &map_ht, bar, kb * BK, 0);
            tma_load_2d_pair(dst + 64 * 128, &map_ht, bar, kb * BK, 0);
          }
        };
        if (RES && prod == 0) {
          // this unit's rows: wait until the previous unit's MMAs released the A region
          if (!warp_wait(aempty_bar, (uint32_t)(ucount & 1) ^ 1u, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) break;
          if (elect_one()) {
            if (leader) mbar_arrive_expect_tx(afull_bar, 2 * a.n_kb * LSE_A_BYTES);
            for (int kb = 0; kb < a.n_kb; ++kb) load_a(abase + kb * LSE_A_BYTES, lead_afull, kb);
            if (!leader) mbar_arrive_cluster(lead_afull);
          }
        }
        for (int vt = vt0; ok && vt < vt1; ++vt) {
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (stage % NPROD == prod) {
              if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
              if (elect_one()) {
                const uint32_t sa = sbase + stage * STAGE_BYTES;
                const uint32_t fb = lead_full0 + 8u * stage;
                if (leader) mbar_arrive_expect_tx(full0 + 8u * stage, 2 * STAGE_BYTES);
                if (!RES) load_a(sa, fb, kb);
                tma_load_2d_pair(sa + (RES ? 0 : LSE_A_BYTES), &map_w, fb, kb * BK,
                                 vt * LSE_BN + (int)rank * (LSE_BN / 2));
                if (!leader) mbar_arrive_cluster(fb);
              }
            }
            ++issued;
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
      }
      if (leader) {
        if (prod == 0) drain_loads<STAGES>(full0, stage, phase, issued);
        if (RES && prod == 0 && ucount > 0) mbar_wait_drain(afull_bar, (uint32_t)((ucount - 1) & 1));
      }
    }
  } else if (warp == 1) {
    if (leader) {
      // ------------------------------------------------------------ pair MMA issuer (leader, whole warp)
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, LSE_BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      int ucount = 0;
      bool ok = true;
      for (int u = cid; ok && u < a.n_units; u += n_clusters, ++ucount) {
        int view, rp, uv, vt0, vt1;
        lse_unit(a, u, view, rp, uv, vt0, vt1);
        if (RES) {
          if (!warp_wait(afull_bar, (uint32_t)(ucount & 1), abort_p, KLG_STATUS_TIMEOUT_MMA)) break;
          tc_fence_after();
        }
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          if (!warp_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + buf * LSE_BN;
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!warp_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
            tc_fence_after();
            if (elect_one()) {
              const uint32_t sa = sbase + stage * STAGE_BYTES;
              const uint32_t a_tile = RES ? abase + kb * LSE_A_BYTES : sa;
              const uint32_t b_tile = RES ? sa : sa + LSE_A_BYTES;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_bf16_pair(d, desc_kmajor(a_tile, k), desc_kmajor(b_tile, k), idesc, (kb | k) != 0);
              mma_commit_pair(empty0 + 8u * stage);
              mma_commit_pair(peer_empty0 + 8u * stage);
            }
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
          if (ok && elect_one()) {
            mma_commit_pair(tfull0 + 8u * buf);
            mma_commit_pair(peer_tfull0 + 8u * buf);
          }
        }
        if (RES && ok && elect_one()) {   // the unit's MMAs are issued: release the A region once they complete
          mma_commit_pair(aempty_bar);
          mma_commit_pair(peer_aempty);
        }
      }
      if (elect_one()) mma_commit_pair(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int h = (warp - EPI_WARP0) >> 2;        // column slice of the 256-column tile
    const int rw = 256 / a.rep;                   // rows per copy
    const int prow = (int)rank * 128 + q * 32;    // the warp's first M row in the pair tile
    const int copy = prow / rw;                   // which copy of the rows these lanes hold
    const int ncol = LSE_BN / (a.rep * LSE_CSPLIT);   // columns per warp and tile (multiple of 32)
    const int slice = (copy * LSE_CSPLIT + h);        // column slice, also the record index
    const int n_slices = a.rep * LSE_CSPLIT;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(slice * ncol);
    int tcount = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int view, rp, uv, vt0, vt1;
      lse_unit(a, u, view, rp, uv, vt0, vt1);
      const int row = rp * 256 + prow % rw + lane;
      const bool live = rp * 256 + prow % rw < a.n_rows;   // warp-uniform
      const uint32_t rk = a.seed_lo ^ ((uint32_t)row * HASH_ROW) ^ (a.seed_hi * HASH_SEED);
      const float thr_row = (EPI == EPI_CAND && live && row < a.n_rows) ? a.thr[row] : INFINITY;
      float m = NEG_BIG, S = 0.f;
      float bk = -INFINITY, bz = 0.f;   // EPI_GREEDY / EPI_SAMPLE: best key, its logit
      int bi = -1;
      for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        if (!mbar_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
        tc_fence_after();
        const int col_base = vt * LSE_BN + slice * ncol;
#pragma unroll 1
        for (int c = 0; live && c < ncol / 32; ++c) {
          uint32_t b0[32];
          tmem_ld32_raw(lane_addr + buf * LSE_BN + c * 32, b0);
          tmem_wait_ld_regs(b0);
          const int nvalid = min(32, a.vocab - (col_base + c * 32));
          if (nvalid > 0) {
            if (EPI == EPI_LSE) {
              lse_chunk(b0, nvalid, a.scale_log2, m, S);
            } else if (EPI == EPI_CAND) {
              // candidates of the filtered sampler: every logit at or above the row's threshold
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float z = __uint_as_float(b0[j]);
                if (j < nvalid && z >= thr_row) {
                  const int slot = atomicAdd(a.cand_cnt + row, 1);
                  if (slot < a.cap) {
                    a.cand_z[(size_t)row * a.cap + slot] = z;
                    a.cand_i[(size_t)row * a.cap + slot] = col_base + c * 32 + j;
                  }
                }
              }
            } else {
              float cmx;
              select_chunk<EPI == EPI_SAMPLE>(b0, nvalid, col_base + c * 32, a.scale_log2, rk, m, S, bk, bi, bz, cmx);
              if (a.cmax && row < a.n_rows) a.cmax[(size_t)row * a.n_ck + (col_base + c * 32) / 32] = cmx;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(tempty0 + 8u * buf);
          else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
        }
      }
      if (ok && row < a.n_rows && EPI != EPI_CAND) {
        if (EPI == EPI_LSE) {
          const size_t n2 = (size_t)a.n_views * a.n_rows;
          float* p = a.parts + ((size_t)(uv * n_slices + slice) * 2) * n2 + (size_t)view * a.n_rows + row;
          p[0] = m;
          p[n2] = S;
        } else {
          const size_t n = (size_t)a.n_rows;
          float* p = a.parts + (size_t)(uv * n_slices + slice) * 5 * n + row;
          p[0] = m;
          p[n] = S;
          p[2 * n] = bk;
          p[3 * n] = __int_as_float(bi);
          p[4 * n] = bz;
        }
      }
    }
  }
  tc_fence_before();
  cluster_sync();   // all pair MMAs retired and both epilogues done before TMEM is released
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, LSE_TMEM_COLS);
}

// =====================================================================================
// pass-2 dZ on CTA pairs
//
// Per unit (256-row pair tile, vocab range of the chunk) the pair recomputes both views'
// logit tiles (M = 256 rows: 128 per CTA, N = 128 vocab: each CTA loads a 64-row half of
// the W tile) into double-buffered TMEM.  8 epilogue warps per CTA (lane quarter x
// 64-column half) form dZ = coef (q - p) as bf16, stage it in shared memory and write it
// with TMA tensor stores; each also accumulates its half of the KL cross term.
// =====================================================================================
// The kernel is load-latency bound (its MMA waits on operands, not on the epilogue), so
// shared memory goes to load stages: dZ leaves through one 32 x 32 staging buffer per
// warp with a TMA store per 32 columns, which leaves room for 5 stages (measured 12 %
// faster than 4 stages with two 32-row staging buffers per warp, and faster than
// st.global from registers).
constexpr int DZP_BN = 128;
constexpr int DZP_STAGES = 5;
constexpr int DZP_B_BYTES = (DZP_BN / 2) * BK * 2;                        // 8 KB
constexpr int DZP_STAGE_BYTES = 2 * TILE_128x64 + DZP_B_BYTES;            // 40 KB
constexpr int DZP_CSPLIT = KLG_EPI_SPLIT;                                 // epilogue warps per lane quarter
constexpr int DZP_EPI_WARPS = 4 * DZP_CSPLIT;
constexpr int DZP_COLS_PER_WARP = DZP_BN / DZP_CSPLIT;                    // 64 or 32
#ifndef KLG_DZ_PROD
#define KLG_DZ_PROD 2
#endif
constexpr int DZP_PROD = KLG_DZ_PROD;                                     // producer warps
constexpr int DZP_PW = EPI_WARP0 + DZP_EPI_WARPS;                         // first extra producer warp
constexpr int DZP_THREADS = 32 * (DZP_PW + DZP_PROD - 1);
// each stage of the ring always belongs to the same producer (stage % DZP_PROD)
constexpr int DZP_STAGING_BYTES = DZP_EPI_WARPS * 32 * 32 * 2;             // per warp: 32 rows x 32 bf16
constexpr int DZP_STORE_COLS = 32;                                        // columns per TMA store box
constexpr int DZP_SMEM = 1024 + DZP_STAGES * DZP_STAGE_BYTES + DZP_STAGING_BYTES + 256;

// Units: n_rt counts 256-row pair tiles; a_parts rows: a_part_base + uv * DZP_CSPLIT + column slice.
// Staging rows are DZP_COLS_PER_WARP bf16 wide (128 or 64 bytes) in the matching TMA swizzle.
enum { MODE_DZ = 0, MODE_STATS = 1 };

// Resident-row variant (RES, H <= 576): the CTA's 128 student rows (up to 9 k-blocks, 144 KB)
// stay in shared memory for a whole unit, so only the teacher rows and the W half stream:
// 12 KB per 256 MMA cycles (47 B/clk/SM) instead of 40 KB per 512 (78 B/clk/SM).  To leave
// room for enough stages beside the resident block, the streamed operands come in
// 32-column sub-blocks (64-byte swizzle), 12 KB a stage.  The resident block is released
// k-block by k-block: the last tile of a unit commits each k-block's release once its MMAs
// retire, and a loader warp (warp 0) refills it with the next unit's rows right away, so a
// unit boundary costs no pipeline drain.
constexpr int DZR_MAX_KB = 9;
constexpr int DZR_SUB = 32;                                   // bf16 per streamed sub-block row (64 B)
constexpr int DZR_HT_BYTES = BM * DZR_SUB * 2;                // 8 KB: 128 teacher rows x 32
constexpr int DZR_W_BYTES = (DZP_BN / 2) * DZR_SUB * 2;       // 4 KB: this CTA's 64 W rows x 32
constexpr int DZR_STAGE_BYTES = DZR_HT_BYTES + DZR_W_BYTES;   // 12 KB
constexpr int DZR_A_BYTES = DZR_MAX_KB * TILE_128x64;         // 144 KB resident student rows
#ifndef KLG_DZR_PROD
#define KLG_DZR_PROD 2
#endif
constexpr int DZR_PROD = KLG_DZR_PROD;                        // streaming producer warps (after the epilogue)
constexpr int DZR_THREADS = 32 * (DZP_PW + DZR_PROD);         // warp 0: resident loader
constexpr int DZR_BAR_BYTES = 512;
template <int MODE>
struct DualResCfg {
  static constexpr int STAGING = MODE == MODE_DZ ? DZP_STAGING_BYTES : 0;
  static constexpr int STAGES_RAW = (227 * 1024 - 1024 - DZR_A_BYTES - STAGING - DZR_BAR_BYTES) / DZR_STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = 1024 + DZR_A_BYTES + STAGES * DZR_STAGE_BYTES + STAGING + DZR_BAR_BYTES;
};

// MODE_DZ: pass 2 (dZ chunk + cross-term partials).  MODE_STATS: the single-pass forward
// for evaluation -- per row and unit the online (m_s, S_s, m_t, S_t, A) record over the
// unit's vocabulary tiles (no dZ, no staging use).
// RES = false: maps h_s, h_t (128 x 64 boxes) and W (64 x 64), 128-byte swizzle.
// RES = true: map_hs as above; map_ht (128 x 32 boxes) and map_w (64 x 32), 64-byte swizzle.
// SPLIT (MODE_DZ, fp32-faithful path): dZ leaves as two bf16 planes, hi through map_out and
// lo = bf16(dZ - hi) through map_out2.
template <int MODE, bool RES, bool SPLIT = false>
__global__ void __launch_bounds__(RES ? DZR_THREADS : DZP_THREADS, 1)
dual_pair_kernel(const __grid_constant__ CUtensorMap map_hs, const __grid_constant__ CUtensorMap map_ht,
               const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_out,
               const __grid_constant__ CUtensorMap map_out2, const DualArgs a) {
  constexpr int STAGES = RES ? DualResCfg<MODE>::STAGES : DZP_STAGES;
  constexpr int STAGE_BYTES = RES ? DZR_STAGE_BYTES : DZP_STAGE_BYTES;
  constexpr int A_REGION = RES ? DZR_A_BYTES : 0;
  constexpr int STAGING = RES ? DualResCfg<MODE>::STAGING : DZP_STAGING_BYTES;
  constexpr int NPROD = RES ? DZR_PROD : DZP_PROD;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t abase = smem_u32(smem);                // resident student rows (RES)
  const uint32_t sbase = abase + A_REGION;              // stage ring
  const uint32_t stg0 = sbase + STAGES * STAGE_BYTES;
  const uint32_t bar0 = stg0 + STAGING;
  const uint32_t full0 = bar0;
  const uint32_t empty0 = bar0 + 8u * STAGES;
  const uint32_t tfull0 = bar0 + 16u * STAGES;
  const uint32_t tempty0 = tfull0 + 16u;
  const uint32_t done_bar = tempty0 + 16u;
  const uint32_t afull0 = done_bar + 8u;                // RES [DZR_MAX_KB]: leader, both CTAs' resident bytes
  const uint32_t aempty0 = afull0 + 8u * DZR_MAX_KB;    // RES [DZR_MAX_KB]: each CTA
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
      mbar_init(tempty0 + 8u * b, 2 * DZP_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    if (RES) {
      for (int kb = 0; kb < DZR_MAX_KB; ++kb) {
        mbar_init(afull0 + 8u * kb, 2);
        mbar_init(aempty0 + 8u * kb, 1);
      }
    }
    fence_mbar_init();
    tma_prefetch(&map_hs);
    tma_prefetch(&map_ht);
    tma_prefetch(&map_w);
    tma_prefetch(&map_out);
    if (SPLIT) tma_prefetch(&map_out2);
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
  const uint32_t lead_afull0 = mapa_shared(afull0, 0);
  const uint32_t peer_empty0 = mapa_shared(empty0, 1);
  const uint32_t peer_tfull0 = mapa_shared(tfull0, 1);
  const uint32_t peer_aempty0 = mapa_shared(aempty0, 1);

  if (RES && warp == 0) {
    // ------------------------------------------------------------ resident loader (both CTAs, whole warp)
    // k-block kb of a unit's student rows is loaded once the previous unit's last tile has
    // retired its MMAs on kb (aempty), so the next unit's rows arrive while that tile finishes.
    int uidx = -1, kb_loaded = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int rt, uv, vt0, vt1;
      dual_unit(a, u, rt, uv, vt0, vt1);
      const int row0 = rt * 256 + (int)rank * 128;
      ++uidx;
      kb_loaded = 0;
      for (int kb = 0; kb < a.n_kb; ++kb) {
        if (!warp_wait(aempty0 + 8u * kb, (uint32_t)(uidx & 1) ^ 1u, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          if (leader) mbar_arrive_expect_tx(afull0 + 8u * kb, 2 * TILE_128x64);
          tma_load_2d_pair(abase + kb * TILE_128x64, &map_hs, lead_afull0 + 8u * kb, kb * BK, row0);
          if (!leader) mbar_arrive_cluster(lead_afull0 + 8u * kb);
        }
        __syncwarp();
        kb_loaded = kb + 1;
      }
    }
    if (leader) {   // every resident load issued has landed (both CTAs' bytes count on the leader)
      for (int kb = 0; kb < a.n_kb; ++kb) {
        const int last = kb < kb_loaded ? uidx : uidx - 1;
        if (last >= 0) mbar_wait_drain(afull0 + 8u * kb, (uint32_t)(last & 1));
      }
    }
  } else if (RES && warp >= DZP_PW) {
    // ------------------------------------------------------------ streaming producers (both CTAs, whole warp)
    // teacher rows and the W half in 32-column sub-blocks; stage s belongs to producer s % NPROD
    const int prod = warp - DZP_PW;
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int rt, uv, vt0, vt1;
      dual_unit(a, u, rt, uv, vt0, vt1);
      const int row0 = rt * 256 + (int)rank * 128;
      for (int vt = vt0; ok && vt < vt1; ++vt) {
        const int wrow = a.v_begin + vt * DZP_BN + (int)rank * (DZP_BN / 2);
        for (int ks = 0; ks < 2 * a.n_kb; ++ks) {
          if (stage % NPROD == prod) {
            if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
            if (elect_one()) {
              const uint32_t sa = sbase + stage * STAGE_BYTES;
              const uint32_t fb = lead_full0 + 8u * stage;
              if (leader) mbar_arrive_expect_tx(full0 + 8u * stage, 2 * STAGE_BYTES);
              tma_load_2d_pair(sa, &map_ht, fb, ks * DZR_SUB, row0);
              tma_load_2d_pair(sa + DZR_HT_BYTES, &map_w, fb, ks * DZR_SUB, wrow);
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
  } else if (!RES && (warp == 0 || warp >= DZP_PW)) {
    // producer warps: warp 0 and warps DZP_PW.. take the pipeline's load steps round-robin
    const int prod = warp == 0 ? 0 : warp - DZP_PW + 1;
    {   // TMA producer (both CTAs, whole warp)
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int rt, uv, vt0, vt1;
        dual_unit(a, u, rt, uv, vt0, vt1);
        const int row0 = rt * 256 + (int)rank * 128;
        for (int vt = vt0; ok && vt < vt1; ++vt) {
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (stage % DZP_PROD == prod) {
              if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
              if (elect_one()) {
                const uint32_t sa = sbase + stage * DZP_STAGE_BYTES;
                const uint32_t fb = lead_full0 + 8u * stage;
                if (leader) mbar_arrive_expect_tx(full0 + 8u * stage, 2 * DZP_STAGE_BYTES);
                tma_load_2d_pair(sa, &map_hs, fb, kb * BK, row0);
                tma_load_2d_pair(sa + TILE_128x64, &map_ht, fb, kb * BK, row0);
                tma_load_2d_pair(sa + 2 * TILE_128x64, &map_w, fb, kb * BK,
                                 a.v_begin + vt * DZP_BN + (int)rank * (DZP_BN / 2));
                if (!leader) mbar_arrive_cluster(fb);
              }
            }
            ++issued;
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
      }
      if (leader && prod == 0) drain_loads<STAGES>(full0, stage, phase, issued);
    }
  } else if (warp == 1) {
    if (leader && RES) {   // pair MMA issuer, resident student rows (leader, whole warp)
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, DZP_BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      int uidx = -1;
      bool ok = true;
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int rt, uv, vt0, vt1;
        dual_unit(a, u, rt, uv, vt0, vt1);
        ++uidx;
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          if (!warp_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_s = tmem + buf * 256;
          const uint32_t d_t = d_s + 128;
          const bool first = vt == vt0, last = vt == vt1 - 1;
          for (int kb = 0; ok && kb < a.n_kb; ++kb) {
            if (first) {   // this unit's k-block kb of the student rows has landed in both CTAs
              if (!warp_wait(afull0 + 8u * kb, (uint32_t)(uidx & 1), abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
              tc_fence_after();
            }
            for (int hf = 0; hf < 2; ++hf) {
              if (!warp_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
              tc_fence_after();
              if (elect_one()) {
                const uint32_t sa = sbase + stage * STAGE_BYTES;
                const uint32_t a_res = abase + kb * TILE_128x64;
#pragma unroll
                for (int j = 0; j < DZR_SUB / 16; ++j) {
                  const uint64_t bdesc = desc_kmajor_sw64(sa + DZR_HT_BYTES, j);
                  const uint32_t acc = (kb | hf | j) != 0;
                  mma_bf16_pair(d_s, desc_kmajor(a_res, 2 * hf + j), bdesc, idesc, acc);
                  mma_bf16_pair(d_t, desc_kmajor_sw64(sa, j), bdesc, idesc, acc);
                }
                mma_commit_pair(empty0 + 8u * stage);
                mma_commit_pair(peer_empty0 + 8u * stage);
              }
              __syncwarp();
              if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
            if (ok && last && elect_one()) {   // the unit's MMAs on kb are issued: release kb once they retire
              mma_commit_pair(aempty0 + 8u * kb);
              mma_commit_pair(peer_aempty0 + 8u * kb);
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
      if (elect_one()) mma_commit_pair(done_bar);
      __syncwarp();
      mbar_wait_drain(done_bar, 0);
    } else if (leader) {   // pair MMA issuer (leader, whole warp)
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, DZP_BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      bool ok = true;
      for (int u = cid; ok && u < a.n_units; u += n_clusters) {
        int rt, uv, vt0, vt1;
        dual_unit(a, u, rt, uv, vt0, vt1);
        for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (tcount >> 1) & 1;
          if (!warp_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_s = tmem + buf * 256;
          const uint32_t d_t = d_s + 128;
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!warp_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
            tc_fence_after();
            if (elect_one()) {
              const uint32_t sa = sbase + stage * DZP_STAGE_BYTES;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k) {
                const uint64_t bdesc = desc_kmajor(sa + 2 * TILE_128x64, k);
                const uint32_t acc = (kb | k) != 0;
                mma_bf16_pair(d_s, desc_kmajor(sa, k), bdesc, idesc, acc);
                mma_bf16_pair(d_t, desc_kmajor(sa + TILE_128x64, k), bdesc, idesc, acc);
              }
              mma_commit_pair(empty0 + 8u * stage);
              mma_commit_pair(peer_empty0 + 8u * stage);
            }
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
          if (ok && elect_one()) {
            mma_commit_pair(tfull0 + 8u * buf);
            mma_commit_pair(peer_tfull0 + 8u * buf);
          }
        }
      }
      if (elect_one()) mma_commit_pair(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else if (MODE == MODE_STATS) {
    // -------------------------------------------------------------- statistics epilogue
    const int q = warp & 3;
    const int h = (warp - EPI_WARP0) >> 2;   // column slice of the 128-column tile
    constexpr int CW = DZP_COLS_PER_WARP;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * CW);
    int tcount = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int rt, uv, vt0, vt1;
      dual_unit(a, u, rt, uv, vt0, vt1);
      const int row = rt * 256 + (int)rank * 128 + q * 32 + lane;
      float ms = NEG_BIG, Ss = 0.f, mt = NEG_BIG, St = 0.f, A = 0.f;
      for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        if (!mbar_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tbase = lane_addr + buf * 256;
#pragma unroll 1
        for (int c = 0; c < CW / 32; ++c) {
          uint32_t bs[32], bt[32];
          tmem_ld32_raw(tbase + c * 32, bs);
          tmem_ld32_raw(tbase + 128 + c * 32, bt);
          tmem_wait_ld_regs(bs, bt);
          const int nvalid = min(32, a.v_count - (vt * DZP_BN + h * CW + c * 32));
          if (nvalid > 0) stats_chunk(bs, bt, nvalid, a.scale_log2, ms, Ss, mt, St, A);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(tempty0 + 8u * buf);
          else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
        }
      }
      if (ok && row < a.n_rows) {
        float* p = a.partials + (size_t)(uv * DZP_CSPLIT + h) * 5 * a.n_rows + row;
        p[0] = ms;
        p[(size_t)a.n_rows] = Ss;
        p[(size_t)2 * a.n_rows] = mt;
        p[(size_t)3 * a.n_rows] = St;
        p[(size_t)4 * a.n_rows] = A;
      }
    }
  } else {
    const int q = warp & 3;
    const int h = (warp - EPI_WARP0) >> 2;   // column slice of the 128-column tile
    constexpr int CW = DZP_COLS_PER_WARP;
    constexpr int NCH = CW / 32;             // 32-column chunks per warp and tile
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * CW);
    const uint32_t stg = stg0 + (uint32_t)(warp - EPI_WARP0) * 2048u;   // this warp's 32 x 32 staging
    const uint64_t pol = l2_evict_first_policy();   // dZ is streamed out once, read by the next kernel
    // 16-byte chunk k of a 64-byte staging row r sits at chunk k ^ ((r / 2) % 4) (64-byte swizzle)
    const uint32_t swz = (uint32_t)((lane >> 1) & 3);
    int tcount = 0;
    bool ok = true;
    for (int u = cid; ok && u < a.n_units; u += n_clusters) {
      int rt, uv, vt0, vt1;
      dual_unit(a, u, rt, uv, vt0, vt1);
      const int row = rt * 256 + (int)rank * 128 + q * 32 + lane;
      const bool row_ok = row < a.n_rows;
      float Ls = 0.f, Lt = 0.f, coef = 0.f, acc = 0.f;
      bool live = false;
      if (row_ok) {
        Ls = a.lse[row];
        Lt = a.lse[a.n_rows + row];
        const float cnt = *a.count;
        const float g = a.grad ? *a.grad : 1.0f;
        live = a.mask[row] && cnt > 0.f;
        coef = live ? g / cnt * a.inv_temp : 0.f;
      }
      for (int vt = vt0; ok && vt < vt1; ++vt, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        if (!mbar_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tbase = lane_addr + buf * 256;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          uint32_t bs[32], bt[32];
          tmem_ld32_raw(tbase + c * 32, bs);
          tmem_ld32_raw(tbase + 128 + c * 32, bt);
          tmem_wait_ld_regs(bs, bt);
          const int nvalid = a.v_count - (vt * DZP_BN + h * CW + c * 32);
          if (SPLIT && nvalid > 0) {
            uint32_t ph[16], pl[16];
            dz_chunk_split(bs, bt, nvalid, a.scale_log2, Ls, Lt, coef, ph, pl, acc);
            const uint32_t rowp = stg + (uint32_t)lane * 64u;
            const int x0 = vt * DZP_BN + h * CW + c * 32, y0 = rt * 256 + (int)rank * 128 + q * 32;
#pragma unroll
            for (int plane = 0; plane < 2; ++plane) {   // the staging buffer serves both planes in turn
              if (lane == 0) bulk_wait_read0();
              __syncwarp();
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t* v = plane ? pl : ph;
                st_shared_v4(rowp + (((uint32_t)k ^ swz) << 4), v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
              }
              fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                if (y0 < a.n_rows) tma_store_2d(plane ? &map_out2 : &map_out, stg, x0, y0);
                bulk_commit();
              }
            }
          } else if (nvalid > 0) {
            uint32_t pk[16];
            dz_chunk(bs, bt, nvalid, a.scale_log2, Ls, Lt, coef, live, pk, acc);
            // staging is free once the previous chunk's store has read it
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            const uint32_t rowp = stg + (uint32_t)lane * 64u;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              st_shared_v4(rowp + (((uint32_t)k ^ swz) << 4), pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
            fence_async_shared();
            __syncwarp();
            const int x0 = vt * DZP_BN + h * CW + c * 32, y0 = rt * 256 + (int)rank * 128 + q * 32;
            if (lane == 0) {
              if (y0 < a.n_rows) tma_store_2d_hint(&map_out, stg, x0, y0, pol);
              bulk_commit();
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(tempty0 + 8u * buf);
          else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
        }
      }
      if (ok && row_ok && a.a_parts)
        a.a_parts[(size_t)(a.a_part_base + uv * DZP_CSPLIT + h) * a.n_rows + row] = acc * a.scale_log2;
    }
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, DUAL_TMEM_COLS);
}

// One GEMM of the backward chunk: C[M][Ncol] (+)= A[M][K] * B[K][Ncol], bf16 in, fp32 out.
// B is MN-major for both problems; A is MN-major for dW (dZ^T) and K-major for dH (dZ).
struct GemmProblem {
  int M, Ncol, K;
  int n_mt, n_nt, n_tiles, n_kb;
  float* C;
  int ldc;
  int accumulate;   // 1: C += A*B, 0: C = A*B
  int a_k0, b_k0;   // K coordinate of the first k-block in A's and B's tensor maps
  int a_mn;         // A stored [K][M] (M contiguous) instead of [M][K]
  int n_split;      // 1, or 2: K split into k-blocks [0, kb_split) and [kb_split, n_kb) (tiles = n_mt*n_nt*n_split)
  int kb_split;
  int c_row0;       // row coordinate of C row 0 in the output tensor map
};

// =====================================================================================
// pair GEMM: the backward chunk's dW = dZ^T h_s and dH (+)= dZ W_chunk in one launch.
// Tile = (problem, 256-row pair tile, BN-column tile); each CTA holds 128 rows of A and
// one BN/2-column half of B (MN-major, 64-byte swizzle: 32-column boxes).  Tiles are
// assigned to pairs by a longest-first greedy schedule built on the host and passed in
// the launch parameters (deterministic; dW tiles are the long ones).
// =====================================================================================
constexpr int PAIR_MAX_TILES = 6144;
constexpr int PAIR_MAX_CLUSTERS = 128;
struct PairSchedule {
  uint32_t tile[PAIR_MAX_TILES];           // tile ids, grouped by pair
  uint16_t start[PAIR_MAX_CLUSTERS + 1];   // pair c runs tile[start[c] .. start[c+1])
};
// Cross-rank dW exchange (row sharding over NVLink, see klg_xr.cuh): problem 0's C tiles are
// not written to C but stored, 32-row block by 32-row block, into the owning rank's inbox.
// Block b of dW (rows 32b .. 32b + 31) belongs to rank b % world, at inbox row
// (b / world) * 32 of slot (src rank, K half) -- [world][2][rows_per_owner][H] fp32 per rank.
constexpr int XR_MAX_WORLD = 8;
struct XrArgs {
  int world;                        // 0: no cross-rank exchange
  int rank;
  int rows_per_owner;               // multiple of 32
  int tma;                          // 1: TMA tensor stores through XrMaps; 0: 16-byte stores from registers
  float* inbox[XR_MAX_WORLD];       // each rank's inbox base (peer pointers)
};
// Tensor maps of every rank's inbox, [2 * world * rows_per_owner][H] fp32, 32 x 32 boxes
// (128-byte swizzle), for the TMA form of the exchange's stores.
struct XrMaps {
  CUtensorMap m[XR_MAX_WORLD];
};
struct PairGemmArgs {
  GemmProblem p[2];   // n_mt counts 256-row pair tiles
  int n_tiles;
  XrArgs xr;
};

#ifndef KLG_GEMM_KPS
#define KLG_GEMM_KPS 1
#endif
template <int BN>
struct PairGemmCfg {
  static constexpr int A_BYTES = TILE_128x64;          // this CTA's 128 rows x 64 K
  static constexpr int B_BYTES = (BN / 2) * BK * 2;    // this CTA's BN/2 columns x 64 K
  // k-blocks per pipeline stage (2 halves the barrier round trips but leaves 3 stages
  // instead of 6, which measured ~9 % slower at the 16k-row shape)
  static constexpr int KPS = KLG_GEMM_KPS;
  static constexpr int STAGE_BYTES = KPS * (A_BYTES + B_BYTES);   // [A kb0 | A kb1 | B kb0 | B kb1]
#ifndef KLG_GEMM_EPI
#define KLG_GEMM_EPI 4
#endif
  // 4 or 8 epilogue warps (8: two per TMEM lane quarter); 8 measured no faster at the
  // 16k-row shape (with one staging buffer per warp) and slower with two (5 load stages)
  static constexpr int EPI_WARPS = KLG_GEMM_EPI;
#ifndef KLG_GEMM_STG_BUFS
#define KLG_GEMM_STG_BUFS 2
#endif
  // per warp: KLG_GEMM_STG_BUFS x (32 rows x 32 fp32); a single buffer would leave room for a
  // 7th stage but serialises the epilogue's reduce-adds (measured 5 % slower)
  static constexpr int STG_BUFS = KLG_GEMM_STG_BUFS;
  static constexpr int STAGING_BYTES = EPI_WARPS * STG_BUFS * 4096;
#ifndef KLG_GEMM_PROD
#define KLG_GEMM_PROD 3
#endif
  static constexpr int PROD = KLG_GEMM_PROD;         // producer warps (each owns stages s % PROD)
  static constexpr int PW = EPI_WARP0 + EPI_WARPS;   // first extra producer warp
  static constexpr int STAGES_RAW = (227 * 1024 - 2048 - STAGING_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int THREADS = 32 * (PW + PROD - 1);
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + 256;
};

__device__ __forceinline__ void pair_tile(const PairGemmArgs& g, int t, int& pi, int& mt, int& nt, int& kb0,
                                          int& kb1) {
  pi = t < g.p[0].n_tiles ? 0 : 1;
  const GemmProblem& P = g.p[pi];
  int lt = pi ? t - g.p[0].n_tiles : t;
  const int split = lt / (P.n_mt * P.n_nt);
  lt -= split * P.n_mt * P.n_nt;
  mt = lt / P.n_nt;
  nt = lt % P.n_nt;
  kb0 = split ? P.kb_split : 0;
  kb1 = (split || P.n_split == 1) ? P.n_kb : P.kb_split;
}

template <int BN>
__global__ void __launch_bounds__(PairGemmCfg<BN>::THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_b0,
                 const __grid_constant__ CUtensorMap map_a1, const __grid_constant__ CUtensorMap map_b1,
                 const __grid_constant__ CUtensorMap map_c0, const __grid_constant__ CUtensorMap map_c1,
                 const PairGemmArgs g, const __grid_constant__ PairSchedule sched,
                 const __grid_constant__ XrMaps xm) {
  using Cfg = PairGemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int EPI = Cfg::EPI_WARPS;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t stg0 = sbase + STAGES * Cfg::STAGE_BYTES;   // epilogue staging (1024-aligned)
  const uint32_t bar0 = stg0 + Cfg::STAGING_BYTES;
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
  const int i0 = sched.start[cid], i1 = sched.start[cid + 1];

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8u * s, 2);
      mbar_init(empty0 + 8u * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8u * b, 1);
      mbar_init(tempty0 + 8u * b, 2 * EPI);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch(&map_a0);
    tma_prefetch(&map_b0);
    tma_prefetch(&map_a1);
    tma_prefetch(&map_b1);
    tma_prefetch(&map_c0);
    tma_prefetch(&map_c1);
  }
  if (warp == 1) tmem_alloc_pair(smem_u32(&tmem_slot), Cfg::TMEM_COLS);
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

  if (warp == 0 || warp >= Cfg::PW) {
    // producer warps: warp 0 and warps Cfg::PW.. take the pipeline's load steps round-robin
    const int prod = warp == 0 ? 0 : warp - Cfg::PW + 1;
    {
      // ------------------------------------------------------------ TMA producer (both CTAs, whole warp)
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int i = i0; ok && i < i1; ++i) {
        int pi, mt, nt, kb0, kb1;
        pair_tile(g, sched.tile[i], pi, mt, nt, kb0, kb1);
        const GemmProblem& P = g.p[pi];
        const CUtensorMap* ma = pi ? &map_a1 : &map_a0;
        const CUtensorMap* mb = pi ? &map_b1 : &map_b0;
        const int row0 = mt * 256 + (int)rank * 128;
        const int col0 = nt * BN + (int)rank * (BN / 2);
        for (int kb = kb0; kb < kb1; kb += Cfg::KPS) {
          const int nk = min(Cfg::KPS, kb1 - kb);
          if (stage % Cfg::PROD == prod) {
            if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) { ok = false; break; }
            if (elect_one()) {
              const uint32_t sa = sbase + stage * Cfg::STAGE_BYTES;
              const uint32_t fb = lead_full0 + 8u * stage;
              if (leader) mbar_arrive_expect_tx(full0 + 8u * stage, 2 * nk * (Cfg::A_BYTES + Cfg::B_BYTES));
              for (int j = 0; j < nk; ++j) {
                const uint32_t saj = sa + j * Cfg::A_BYTES;
                const uint32_t sbj = sa + Cfg::KPS * Cfg::A_BYTES + j * Cfg::B_BYTES;
                const int ka = P.a_k0 + (kb + j) * BK, kbb = P.b_k0 + (kb + j) * BK;
                if (P.a_mn) {
                  tma_load_2d_pair(saj, ma, fb, row0, ka);
                  tma_load_2d_pair(saj + 8192, ma, fb, row0 + 64, ka);
                } else {
                  tma_load_2d_pair(saj, ma, fb, ka, row0);
                }
  #pragma unroll
                for (int jj = 0; jj < BN / 64; ++jj) tma_load_2d_pair(sbj + 4096 * jj, mb, fb, col0 + 32 * jj, kbb);
              }
              if (!leader) mbar_arrive_cluster(fb);
            }
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (leader && prod == 0) drain_loads<STAGES>(full0, stage, phase, issued);
    }
  } else if (warp == 1) {
    if (leader) {
      // ------------------------------------------------------------ pair MMA issuer (leader, whole warp)
      constexpr uint32_t idesc_kmaj = make_idesc_bf16(2 * BM, BN, false, true);
      constexpr uint32_t idesc_mnmaj = make_idesc_bf16(2 * BM, BN, true, true);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = i0, k = 0; ok && i < i1; ++i, ++k) {
        int pi, mt, nt, kb0, kb1;
        pair_tile(g, sched.tile[i], pi, mt, nt, kb0, kb1);
        const GemmProblem& P = g.p[pi];
        const bool amn = P.a_mn != 0;
        const uint32_t idesc = amn ? idesc_mnmaj : idesc_kmaj;
        const int buf = k & 1;
        const uint32_t tph = (uint32_t)(k >> 1) & 1u;
        if (!warp_wait(tempty0 + 8u * buf, tph ^ 1, abort_p, KLG_STATUS_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = kb0; kb < kb1; kb += Cfg::KPS) {
          const int nk = min(Cfg::KPS, kb1 - kb);
          if (!warp_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          if (elect_one()) {
            const uint32_t sa = sbase + stage * Cfg::STAGE_BYTES;
            for (int j = 0; j < nk; ++j) {
              const uint32_t saj = sa + j * Cfg::A_BYTES;
              const uint32_t sbj = sa + Cfg::KPS * Cfg::A_BYTES + j * Cfg::B_BYTES;
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk) {
                const uint64_t ad = amn ? desc_mnmajor(saj, kk) : desc_kmajor(saj, kk);
                mma_bf16_pair(d, ad, desc_mnmajor_sw64(sbj, kk), idesc, (kb + j > kb0 || kk > 0) ? 1u : 0u);
              }
            }
            mma_commit_pair(empty0 + 8u * stage);
            mma_commit_pair(peer_empty0 + 8u * stage);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok && elect_one()) {
          mma_commit_pair(tfull0 + 8u * buf);
          mma_commit_pair(peer_tfull0 + 8u * buf);
        }
      }
      if (elect_one()) mma_commit_pair(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    // Each 32 x 32 fp32 block goes through a 128-byte-swizzled staging buffer and is added
    // into C by a TMA reduce-add (the add happens at L2), or stored when the problem's
    // accumulate flag is 0 (the tile's first and only addend in C).
    const int q = warp & 3;
    const int hh = (warp - EPI_WARP0) >> 2;          // column half when two warps share a quarter
    constexpr int PER = (BN / 32) / (EPI / 4);       // 32-column blocks per warp and tile
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t stg = stg0 + (uint32_t)(warp - EPI_WARP0) * (Cfg::STG_BUFS * 4096u);
    int sbuf = 0;
    for (int i = i0, k = 0; i < i1; ++i, ++k) {
      int pi, mt, nt, kb0, kb1;
      pair_tile(g, sched.tile[i], pi, mt, nt, kb0, kb1);
      const GemmProblem& P = g.p[pi];
      const CUtensorMap* mc = pi ? &map_c1 : &map_c0;
      const int buf = k & 1;
      const uint32_t tph = (uint32_t)(k >> 1) & 1u;
      if (!mbar_wait(tfull0 + 8u * buf, tph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const int row_blk = mt * 256 + (int)rank * 128 + q * 32;   // first C row of this warp
#pragma unroll 1
      for (int c = hh * PER; c < (hh + 1) * PER; ++c) {
        uint32_t v[32];
        tmem_ld32_raw(lane_addr + buf * BN + c * 32, v);
        tmem_wait_ld_regs(v);
        const int col0 = nt * BN + c * 32;
        if (row_blk >= P.M || col0 >= P.Ncol) continue;   // warp-uniform
        const bool xr_blk = pi == 0 && g.xr.world > 0;
        const int xr_vb = P.c_row0 + row_blk;            // first dW row of this 32-row block (multiple of 32)
        const int xr_owner = xr_blk ? (xr_vb >> 5) % g.xr.world : 0;
        const int xr_row = xr_blk ? (g.xr.rank * 2 + (kb0 > 0 ? 1 : 0)) * g.xr.rows_per_owner +
                                        ((xr_vb >> 5) / g.xr.world) * 32
                                  : 0;                   // inbox row of the block: slot (rank, K half), owner's row
        if (xr_blk && !g.xr.tma) {
          // dW block to its owner's inbox (plain 16-byte stores over NVLink, no atomics): rows
          // past M are not written; the K half (split tiles) picks the slot
          const int owner = xr_owner;
          const int orow = ((xr_vb >> 5) / g.xr.world) * 32 + lane;
          const int slot = g.xr.rank * 2 + (kb0 > 0 ? 1 : 0);
          // columns past Ncol (H not a multiple of 32) are not written either: H % 8 == 0, so the
          // block's valid columns are whole float4s
          const int n4 = min(8, (P.Ncol - col0) >> 2);
          if (row_blk + lane < P.M) {
            float4* dst = reinterpret_cast<float4*>(g.xr.inbox[owner] +
                                                    ((size_t)slot * g.xr.rows_per_owner + orow) * P.ldc + col0);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (j < n4)
                dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                     __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
          }
          continue;
        }
        if (lane == 0) {                                   // the buffer written STG_BUFS blocks ago is free
          if (Cfg::STG_BUFS == 2) bulk_wait_read1();
          else bulk_wait_read0();
        }
        __syncwarp();
        const uint32_t rowp = stg + (uint32_t)sbuf * 4096u + (uint32_t)lane * 128u;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(rowp + (((uint32_t)j ^ (uint32_t)(lane & 7)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                       v[4 * j + 3]);
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (xr_blk) tma_store_2d(&xm.m[xr_owner], stg + (uint32_t)sbuf * 4096u, col0, xr_row);   // owner's inbox
          else if (P.accumulate) tma_reduce_add_2d(mc, stg + (uint32_t)sbuf * 4096u, col0, P.c_row0 + row_blk);
          else tma_store_2d(mc, stg + (uint32_t)sbuf * 4096u, col0, P.c_row0 + row_blk);
          bulk_commit();
        }
        sbuf = (sbuf + 1) % Cfg::STG_BUFS;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(tempty0 + 8u * buf);
        else mbar_arrive_cluster(lead_tempty0 + 8u * buf);
      }
    }
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
}

// =====================================================================================
// small kernels
// =====================================================================================

// count = sum(mask), one block, deterministic.
__global__ void count_valid_kernel(const uint8_t* __restrict__ mask, int n, float* __restrict__ count) {
  pdl_enter();
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
  pdl_enter();
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
  pdl_enter();
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

// Merge of n_part (m, S) records parts[n_part][2][n2] (log2 units) per row i: lse[i] = the
// log-sum-exp (when lse is set) and/or rec = the merged record [2][n2] (when rec is set; a
// vocab shard's record, to be gathered with the other shards' and merged again).
// With count or done set, the grid has one block more than the rows need: that block writes
// *count = sum(mask[0..n_rows)) (fixed order) when count is set and clears *done (the loss
// kernel's completion counter) when done is set.
__global__ void lse_merge_kernel(const float* __restrict__ parts, int n_part, int n2, float* __restrict__ lse,
                                 float* __restrict__ rec, const uint8_t* __restrict__ mask, int n_rows,
                                 float* __restrict__ count, unsigned* __restrict__ done) {
  pdl_enter();
  if ((count || done) && blockIdx.x == gridDim.x - 1) {
    __shared__ int part[32];
    if (count) {
      int c = 0;
      for (int r = threadIdx.x; r < n_rows; r += blockDim.x) c += mask[r] != 0;
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
    if (done && threadIdx.x == 0) *done = 0u;
    return;
  }
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n2) return;
  const size_t st = (size_t)n2;
  float M = NEG_BIG;
  for (int p = 0; p < n_part; ++p) M = fmaxf(M, parts[(size_t)p * 2 * st + i]);
  float S = 0.f;
  for (int p = 0; p < n_part; ++p) S = fmaf(parts[(size_t)p * 2 * st + st + i], ex2(parts[(size_t)p * 2 * st + i] - M), S);
  if (lse) lse[i] = M + __log2f(S);
  if (rec) {
    rec[i] = M;
    rec[st + i] = S;
  }
}

// cross[i] = sum over the pass-2 partial rows a_parts[p][i] in a fixed order: the KL cross
// term sum_v p_v (u_t - u_s) (log2 units) of row i over the vocabulary the pass covered.
__global__ void cross_sum_kernel(const float* __restrict__ a_parts, int n_ap, int n, float* __restrict__ cross) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float A = 0.f;
  for (int p = 0; p < n_ap; ++p) A += a_parts[(size_t)p * n + i];
  cross[i] = A;
}

// Loss from complete cross terms (e.g. summed over vocab shards): KL_i = ln2 (cross_i + L_s,i -
// L_t,i) for rows with mask set (0 elsewhere), loss = sum KL / count (0 when count == 0).  One
// block; fixed reduction order.
__global__ void kl_loss_kernel(const float* __restrict__ lse, const float* __restrict__ cross,
                               const uint8_t* __restrict__ mask, int n, const float* __restrict__ count,
                               float* __restrict__ loss, float* __restrict__ row_kl) {
  pdl_enter();
  __shared__ float part[32];
  const float ln2 = 0.69314718055994530942f;
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float kl = mask[i] ? ln2 * (cross[i] + lse[i] - lse[(size_t)n + i]) : 0.f;
    if (row_kl) row_kl[i] = kl;
    acc += kl;
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

// lm_head selection: merge the per-unit records (m, S, key, index, z) of each row into the
// chosen token (highest key, lowest index among equals), its logit and the natural-log
// log-sum-exp of z / T (so p(token) = exp(z_token / T - lse)).  A block takes 32 rows (one
// per lane, coalesced loads) and the records of group blockIdx.y (gridDim.y groups); its
// warps take the group's records round-robin and combine through shared memory.  With
// out_parts set, each group writes one merged record [gridDim.y][5][N] for a second launch
// (one group) to finish: a few rows with hundreds of records are then not a serial chain
// of loads on one SM.
#ifndef KLG_SMERGE_WARPS
#define KLG_SMERGE_WARPS 16
#endif
constexpr int SMERGE_WARPS = KLG_SMERGE_WARPS;
__device__ __forceinline__ void merge_best(float k, int idx, float z, float& bk, int& bi, float& bz) {
  const bool take = idx >= 0 && (k > bk || (k == bk && idx < bi));
  bk = take ? k : bk;
  bi = take ? idx : bi;
  bz = take ? z : bz;
}

__global__ void __launch_bounds__(SMERGE_WARPS * 32)
sample_merge_kernel(const float* __restrict__ parts, int n_part, int n, float* __restrict__ out_parts,
                    int* __restrict__ tokens, float* __restrict__ logit, float* __restrict__ lse) {
  pdl_enter();
  __shared__ float sm_m[SMERGE_WARPS][32], sm_s[SMERGE_WARPS][32], sm_k[SMERGE_WARPS][32], sm_z[SMERGE_WARPS][32];
  __shared__ int sm_i[SMERGE_WARPS][32];
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;
  const size_t st = (size_t)n;
  float M = NEG_BIG, S = 0.f, bk = -INFINITY, bz = 0.f;
  int bi = -1;
  const int per = (n_part + gridDim.y - 1) / gridDim.y;
  const int p0 = blockIdx.y * per;
  const int p1 = min(n_part, p0 + per);
  if (i < n) {
#pragma unroll 4
    for (int p = p0 + w; p < p1; p += SMERGE_WARPS) {
      const float* r = parts + (size_t)p * 5 * st + i;
      const float m = r[0], s = r[st], k = r[2 * st], z = r[4 * st];
      const int idx = __float_as_int(r[3 * st]);
      const float nm = fmaxf(M, m);
      S = fmaf(S, ex2(M - nm), s * ex2(m - nm));
      M = nm;
      merge_best(k, idx, z, bk, bi, bz);
    }
  }
  sm_m[w][lane] = M;
  sm_s[w][lane] = S;
  sm_k[w][lane] = bk;
  sm_i[w][lane] = bi;
  sm_z[w][lane] = bz;
  __syncthreads();
  if (w == 0 && i < n) {
    for (int v = 1; v < SMERGE_WARPS; ++v) {
      const float m = sm_m[v][lane];
      const float nm = fmaxf(M, m);
      S = fmaf(S, ex2(M - nm), sm_s[v][lane] * ex2(m - nm));
      M = nm;
      merge_best(sm_k[v][lane], sm_i[v][lane], sm_z[v][lane], bk, bi, bz);
    }
    if (out_parts) {
      float* o = out_parts + (size_t)blockIdx.y * 5 * st + i;
      o[0] = M;
      o[st] = S;
      o[2 * st] = bk;
      o[3 * st] = __int_as_float(bi);
      o[4 * st] = bz;
    } else {
      tokens[i] = bi;
      logit[i] = bz;
      lse[i] = (M + __log2f(S)) * 0.69314718055994530942f;
    }
  }
}

// ---------------------------------------------------------------- filtered sampling (top-k / top-p)
// Order-preserving 32-bit keys of floats (a larger float has a larger key), and back.
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

constexpr int FILT_THREADS = 256;

template <typename T>
__device__ __forceinline__ T block_sum(T v, T* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();   // red is free (a previous call's readers are done)
  if (lane == 0) red[w] = v;
  __syncthreads();
  T t = 0;
#pragma unroll
  for (int i = 0; i < FILT_THREADS / 32; ++i) t += red[i];
  return t;
}

// Per row (one block): a threshold below which no logit survives top-k / top-p, from the
// row's 32-column chunk maxima c (raw logits) and its log-sum-exp lse (natural log, of z / T).
//  top-k: the k-th largest chunk maximum -- the k chunks holding the largest maxima give k
//         logits at or above it, so the k-th largest logit is too;
//  top-p: the largest chunk maximum c* whose chunk maxima at or above it carry softmax mass
//         > top_p -- the logits at or above c* then carry more than top_p, so every logit
//         below c* has more than top_p of mass above it and top-p removes it.
// thr[row] = the top-k bound when top-k is on -- top-p then renormalises over the top-k set,
// all of which must be among the candidates -- else the top-p bound (-inf when neither
// applies).  Both are found by a bit-by-bit search over the order-preserving keys (32
// block-wide passes).
__global__ void __launch_bounds__(FILT_THREADS) filter_threshold_kernel(const float* __restrict__ cmax, int n_ck,
                                                                        const float* __restrict__ lse, float inv_temp,
                                                                        int top_k, float top_p,
                                                                        float* __restrict__ thr) {
  pdl_enter();
  __shared__ double redd[FILT_THREADS / 32];
  __shared__ int redi[FILT_THREADS / 32];
  const int row = blockIdx.x;
  const float* c = cmax + (size_t)row * n_ck;
  const float L = lse[row];
  float tk = -INFINITY, tp = -INFINITY;
  if (top_k > 0 && top_k <= n_ck) {
    uint32_t T = 0;
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t cand = T | (1u << bit);
      int cnt = 0;
      for (int i = threadIdx.x; i < n_ck; i += FILT_THREADS) cnt += fkey(c[i]) >= cand;
      if (block_sum(cnt, redi) >= top_k) T = cand;
    }
    tk = fkey_value(T);
  }
  if (top_k == 0 && top_p < 1.f) {
    auto mass_at_or_above = [&](uint32_t T) {
      double m = 0.0;
      for (int i = threadIdx.x; i < n_ck; i += FILT_THREADS)
        if (fkey(c[i]) >= T) m += exp((double)c[i] * inv_temp - (double)L);
      return block_sum(m, redd);
    };
    if (mass_at_or_above(0u) > (double)top_p) {
      uint32_t T = 0;
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = T | (1u << bit);
        if (mass_at_or_above(cand) > (double)top_p) T = cand;
      }
      tp = fkey_value(T);
    }
  }
  if (threadIdx.x == 0) thr[row] = top_k > 0 ? tk : tp;
}

// Per row (one block): the filtered draw from the candidates (every logit >= the row's
// threshold, so a superset of what top-k / top-p keep).  top-k keeps the candidates at or
// above the k-th largest value (ties stay, as generate.py:61); top-p keeps a candidate when
// the softmax mass strictly above it (over the top-k survivors, or over the whole row when
// top_k = 0, whose mass is exp(z / T - lse)) is <= top_p (generate.py:64-73: the shifted
// removal keeps the entry that crosses top_p).  The token is the Gumbel-max draw over the
// kept candidates with the same keys as the unfiltered sampler (hash of seed, row, column);
// lse_out is log sum exp(z / T) over the kept entries, so p(token) = exp(z / T - lse_out)
// -- the reference's renormalised probability.  A row with more candidates than the list
// holds sets *overflow and gets token -1.
__global__ void __launch_bounds__(FILT_THREADS) filter_select_kernel(
    const int* __restrict__ cand_cnt, const float* __restrict__ cand_z, const int* __restrict__ cand_i, int cap,
    const float* __restrict__ lse, float inv_temp, int top_k, float top_p, uint32_t seed_lo, uint32_t seed_hi,
    int32_t* __restrict__ tokens, float* __restrict__ logit, float* __restrict__ lse_out, int* __restrict__ overflow) {
  pdl_enter();
  __shared__ double redd[FILT_THREADS / 32];
  __shared__ int redi[FILT_THREADS / 32];
  __shared__ float redf[FILT_THREADS / 32];
  __shared__ uint32_t redk[FILT_THREADS / 32];
  const int row = blockIdx.x;
  const int total = cand_cnt[row];
  if (total > cap) {
    if (threadIdx.x == 0) {
      atomicOr(overflow, 1);
      tokens[row] = -1;
      logit[row] = __int_as_float(0x7fc00000);
      lse_out[row] = __int_as_float(0x7fc00000);
    }
    return;
  }
  const int n = total;
  const float* z = cand_z + (size_t)row * cap;
  const int* ix = cand_i + (size_t)row * cap;
  const double L = lse[row];
  // top-k: the k-th largest candidate value's key
  uint32_t Tk = 0;
  if (top_k > 0 && top_k <= n) {
    uint32_t T = 0;
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t cand = T | (1u << bit);
      int cnt = 0;
      for (int i = threadIdx.x; i < n; i += FILT_THREADS) cnt += fkey(z[i]) >= cand;
      if (block_sum(cnt, redi) >= top_k) T = cand;
    }
    Tk = T;
  }
  // softmax weights of the entries top-p measures: over the top-k survivors, or the whole row
  double mref = L, Z = 1.0;
  if (top_k > 0) {
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += FILT_THREADS)
      if (fkey(z[i]) >= Tk) mx = fmaxf(mx, z[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) redf[threadIdx.x >> 5] = mx;
    __syncthreads();
    for (int i = 0; i < FILT_THREADS / 32; ++i) mx = fmaxf(mx, redf[i]);
    mref = (double)mx * inv_temp;
    double zs = 0.0;
    for (int i = threadIdx.x; i < n; i += FILT_THREADS)
      if (fkey(z[i]) >= Tk) zs += exp((double)z[i] * inv_temp - mref);
    Z = block_sum(zs, redd);
  }
  // top-p: keep key >= Tp, Tp = 1 + the largest T whose strictly-larger mass exceeds top_p
  uint32_t Tp = 0;
  if (top_p < 1.f) {
    auto mass_above = [&](uint32_t T) {
      double m = 0.0;
      for (int i = threadIdx.x; i < n; i += FILT_THREADS) {
        const uint32_t k = fkey(z[i]);
        if (k > T && k >= Tk) m += exp((double)z[i] * inv_temp - mref);
      }
      return block_sum(m, redd) / Z;
    };
    if (mass_above(0u) > (double)top_p) {
      uint32_t T = 0;
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = T | (1u << bit);
        if (mass_above(cand) > (double)top_p) T = cand;
      }
      Tp = T + 1;
    }
  }
  const uint32_t Tkeep = Tk > Tp ? Tk : Tp;
  // Gumbel-max over the kept candidates (lowest column among equal keys), and their lse
  const float sl2 = inv_temp * 1.4426950408889634f;
  float bk = -INFINITY, bz = 0.f, mk = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += FILT_THREADS) {
    if (fkey(z[i]) < Tkeep) continue;
    const int col = ix[i];
    const float key = fmaf(z[i], sl2, -__log2f(exp_variate_log2(sample_hash(seed_lo, seed_hi, (uint32_t)row, (uint32_t)col))));
    if (key > bk || (key == bk && col < bi)) {
      bk = key;
      bi = col;
      bz = z[i];
    }
    mk = fmaxf(mk, z[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    const float oz = __shfl_xor_sync(0xffffffffu, bz, o);
    if (ok > bk || (ok == bk && oi < bi)) {
      bk = ok;
      bi = oi;
      bz = oz;
    }
    mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    redf[threadIdx.x >> 5] = bk;
    redi[threadIdx.x >> 5] = bi;
    redk[threadIdx.x >> 5] = __float_as_uint(bz);
    redd[threadIdx.x >> 5] = mk;
  }
  __syncthreads();
  bk = -INFINITY;
  bi = 0x7fffffff;
  bz = 0.f;
  mk = -INFINITY;
  for (int w = 0; w < FILT_THREADS / 32; ++w) {
    if (redf[w] > bk || (redf[w] == bk && redi[w] < bi)) {
      bk = redf[w];
      bi = redi[w];
      bz = __uint_as_float(redk[w]);
    }
    mk = fmaxf(mk, (float)redd[w]);
  }
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += FILT_THREADS)
    if (fkey(z[i]) >= Tkeep) ss += exp((double)(z[i] - mk) * inv_temp);
  ss = block_sum(ss, redd);
  if (threadIdx.x == 0) {
    tokens[row] = bi == 0x7fffffff ? -1 : bi;
    logit[row] = bz;
    lse_out[row] = (float)((double)mk * inv_temp + log(ss));
  }
}

// Training-path per-row KL: KL_i = ln2 * (sum_p a_parts[p][i] + L_s,i - L_t,i) for rows
// carrying loss (0 elsewhere).  Each block writes the sum of its rows' masked KL to
// block_sums[blockIdx.x]; the block that finishes last (counted on *done, which starts at 0
// and is left at 0) forms loss = sum(block_sums) / count in a fixed order (0 when count == 0).
__global__ void row_kl_pair_kernel(const float* __restrict__ lse, const float* __restrict__ a_parts, int n_ap,
                                   const uint8_t* __restrict__ mask, int n, float* __restrict__ row_kl,
                                   float* __restrict__ block_sums, const float* __restrict__ count,
                                   float* __restrict__ loss, unsigned* __restrict__ done) {
  pdl_enter();
  __shared__ float part[8];
  __shared__ bool last;
  const float ln2 = 0.69314718055994530942f;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float kl = 0.f;
  if (i < n && mask[i]) {
    float A = 0.f;
    for (int p = 0; p < n_ap; ++p) A += a_parts[(size_t)p * n + i];
    kl = ln2 * (A + lse[i] - lse[(size_t)n + i]);
  }
  if (row_kl && i < n) row_kl[i] = kl;
  float acc = kl;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    block_sums[blockIdx.x] = t;
    __threadfence();
    last = atomicAdd(done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float tot = 0.f;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) tot += __ldcg(block_sums + b);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  __syncthreads();   // part[] is reused
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = tot;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    const float c = *count;
    *loss = c > 0.f ? t / c : 0.f;
    *done = 0u;
  }
}


// Self-test of the bounded wait: one warp waits on an mbarrier that nothing arrives on.
// mbar_wait gives up after KLG_WAIT_CYCLES, sets KLG_STATUS_SELFTEST and returns false.
__global__ void wait_selftest_kernel() {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  (void)warp_wait(smem_u32(&bar), 0, &abort_flag, KLG_STATUS_SELFTEST);
}

// Zero n floats (n % 4 == 0, 16-byte aligned): gradient buffers before pass 2's reduce-adds.
__global__ void zero_f32x4_kernel(float4* __restrict__ p, long long n4) {
  pdl_enter();
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) p[i] = z;
}

// ---------------------------------------------------------------- row selection (train.py:124-164)
// One warp per selected row i = (b, blk, k), k = 1..K-1: student row b*(nb*K) + blk*K + k of
// diff, teacher row b*L + clamp(anchor[b, blk] + k - 1, 0, L - 1) of ar, valid = target of the
// student position != pad.  Rows are copied as bytes (any dtype; row_bytes % 16 == 0).
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint8_t* __restrict__ diff,
                                                          const uint8_t* __restrict__ ar,
                                                          const long long* __restrict__ anchors,
                                                          const long long* __restrict__ targets, int B, int nb,
                                                          int K, int L, int row_bytes, long long pad,
                                                          uint8_t* __restrict__ hs, uint8_t* __restrict__ ht,
                                                          uint8_t* __restrict__ valid) {
  pdl_enter();
  const int n = nb * (K - 1);
  const long long i = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= (long long)B * n) return;
  const int b = (int)(i / n);
  const int j = (int)(i - (long long)b * n);
  const int blk = j / (K - 1);
  const int k = j - blk * (K - 1) + 1;
  const long long srow = (long long)b * nb * K + (long long)blk * K + k;
  long long t = anchors[(size_t)b * nb + blk] + k - 1;
  t = t < 0 ? 0 : (t > L - 1 ? L - 1 : t);
  const long long trow = (long long)b * L + t;
  if (lane == 0) valid[i] = targets[srow] != pad ? 1 : 0;
  const uint4* s4 = reinterpret_cast<const uint4*>(diff + srow * row_bytes);
  const uint4* t4 = reinterpret_cast<const uint4*>(ar + trow * row_bytes);
  uint4* hs4 = reinterpret_cast<uint4*>(hs + i * row_bytes);
  uint4* ht4 = reinterpret_cast<uint4*>(ht + i * row_bytes);
  for (int c = lane; c < row_bytes / 16; c += 32) {
    hs4[c] = s4[c];
    ht4[c] = t4[c];
  }
}

// Backward of the student selection: every diff position (b, p) gets the gradient row of its
// selected row, or zeros at the anchors (p % K == 0), which carry no loss.
__global__ void __launch_bounds__(256) scatter_rows_grad_kernel(const uint8_t* __restrict__ dhs, int B, int nb, int K,
                                                                int row_bytes, uint8_t* __restrict__ ddiff) {
  pdl_enter();
  const long long p = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p >= (long long)B * nb * K) return;
  const int b = (int)(p / ((long long)nb * K));
  const int pos = (int)(p - (long long)b * nb * K);
  const int k = pos % K;
  uint4* d4 = reinterpret_cast<uint4*>(ddiff + p * row_bytes);
  if (k == 0) {
    for (int c = lane; c < row_bytes / 16; c += 32) d4[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const long long i = (long long)b * nb * (K - 1) + (long long)(pos / K) * (K - 1) + k - 1;
  const uint4* s4 = reinterpret_cast<const uint4*>(dhs + i * row_bytes);
  for (int c = lane; c < row_bytes / 16; c += 32) d4[c] = s4[c];
}

// ---------------------------------------------------------------- final RMSNorm (pre-norm inputs)
// The backbone's final norm (LlamaRMSNorm): r = 1 / sqrt(mean_k x_k^2 + eps) in fp32, and
// bf16 rows  y = bf16(gamma * bf16(x r))  for bf16 x (the norm's own rounding to the input
// dtype, then a bf16 product), y = bf16(gamma * (x r)) for fp32 x (the fp32 norm output,
// rounded once for the GEMM).  One warp per row, 16-byte vector loads (H % 8 == 0).
__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <bool F32>
__device__ __forceinline__ void load8(const void* __restrict__ x, size_t off, float (&v)[8]) {
  if (F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + off);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + off);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

template <bool F32>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const void* __restrict__ x, const float* __restrict__ gamma,
                                                           int n, int hidden, float eps,
                                                           __nv_bfloat16* __restrict__ y, float* __restrict__ rstd) {
  pdl_enter();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const size_t base = (size_t)row * hidden;
  float ss = 0.f;
  for (int c = lane * 8; c < hidden; c += 256) {
    float v[8];
    load8<F32>(x, base + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
  }
  ss = warp_sum_f32(ss);
  const float r = 1.0f / sqrtf(ss / (float)hidden + eps);
  for (int c = lane * 8; c < hidden; c += 256) {
    float v[8];
    load8<F32>(x, base + c, v);
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = v[2 * j] * r, b = v[2 * j + 1] * r;
      if (!F32) {
        a = __bfloat162float(__float2bfloat16_rn(a));
        b = __bfloat162float(__float2bfloat16_rn(b));
      }
      const __nv_bfloat162 t = __floats2bfloat162_rn(g[2 * j] * a, g[2 * j + 1] * b);
      o[j] = *reinterpret_cast<const uint32_t*>(&t);
    }
    *reinterpret_cast<uint4*>(y + base + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (rstd && lane == 0) rstd[row] = r;
}

// Gradient through the norm (the roundings pass the gradient through unchanged, as
// autograd's dtype casts do):  dx_k = r gamma_k dy_k - (r^3 / H) x_k sum_j gamma_j dy_j x_j.
template <bool F32>
__global__ void __launch_bounds__(256) rmsnorm_rows_bwd_kernel(const void* __restrict__ x,
                                                               const float* __restrict__ gamma,
                                                               const float* __restrict__ rstd,
                                                               const float* __restrict__ dy, int n, int hidden,
                                                               float* __restrict__ dx) {
  pdl_enter();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const size_t base = (size_t)row * hidden;
  float s = 0.f;
  for (int c = lane * 8; c < hidden; c += 256) {
    float v[8];
    load8<F32>(x, base + c, v);
    const float4 d0 = *reinterpret_cast<const float4*>(dy + base + c);
    const float4 d1 = *reinterpret_cast<const float4*>(dy + base + c + 4);
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
    s = fmaf(g0.x * d0.x, v[0], s); s = fmaf(g0.y * d0.y, v[1], s);
    s = fmaf(g0.z * d0.z, v[2], s); s = fmaf(g0.w * d0.w, v[3], s);
    s = fmaf(g1.x * d1.x, v[4], s); s = fmaf(g1.y * d1.y, v[5], s);
    s = fmaf(g1.z * d1.z, v[6], s); s = fmaf(g1.w * d1.w, v[7], s);
  }
  s = warp_sum_f32(s);
  const float r = rstd[row];
  const float c3 = r * r * r * s / (float)hidden;
  for (int c = lane * 8; c < hidden; c += 256) {
    float v[8];
    load8<F32>(x, base + c, v);
    const float4 d0 = *reinterpret_cast<const float4*>(dy + base + c);
    const float4 d1 = *reinterpret_cast<const float4*>(dy + base + c + 4);
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
    float4 o0, o1;
    o0.x = fmaf(r * g0.x, d0.x, -c3 * v[0]); o0.y = fmaf(r * g0.y, d0.y, -c3 * v[1]);
    o0.z = fmaf(r * g0.z, d0.z, -c3 * v[2]); o0.w = fmaf(r * g0.w, d0.w, -c3 * v[3]);
    o1.x = fmaf(r * g1.x, d1.x, -c3 * v[4]); o1.y = fmaf(r * g1.y, d1.y, -c3 * v[5]);
    o1.z = fmaf(r * g1.z, d1.z, -c3 * v[6]); o1.w = fmaf(r * g1.w, d1.w, -c3 * v[7]);
    *reinterpret_cast<float4*>(dx + base + c) = o0;
    *reinterpret_cast<float4*>(dx + base + c + 4) = o1;
  }
}

// ---------------------------------------------------------------- logit of a given token
// z[i] = h[i] . W[tokens[i]] in fp32 from bf16 rows (one warp per row, 16-byte loads): the
// logit the fused sampler never writes out, for a token chosen elsewhere.
__global__ void __launch_bounds__(256) token_logit_kernel(const __nv_bfloat16* __restrict__ h,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const int* __restrict__ tokens, int n, int hidden, int vocab,
                                                          float* __restrict__ z) {
  pdl_enter();
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int t = tokens[i];
  float acc = 0.f;
  if (t >= 0 && t < vocab) {
    const size_t hr = (size_t)i * hidden, wr = (size_t)t * hidden;
    for (int c = lane * 8; c < hidden; c += 256) {
      float a[8], b[8];
      load8<false>(h, hr + c, a);
      load8<false>(w, wr + c, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = fmaf(a[j], b[j], acc);
    }
  }
  acc = warp_sum_f32(acc);
  if (lane == 0) z[i] = (t >= 0 && t < vocab) ? acc : __int_as_float(0x7fc00000);   // NaN for a token out of range
}

// fp32 rows -> bf16 rows three times as wide, for the fp32-faithful path: with hi = bf16(x)
// and lo = bf16(x - hi), row r of out is [hi | hi | lo] (order 0, the hidden states) or
// [hi | lo | hi] (order 1, the lm_head), so the products of the two kinds of rows along the
// 3H columns add up to x_hi w_hi + x_hi w_lo + x_lo w_hi.
__global__ void split3_kernel(const float* __restrict__ x, long long n_rows, int hidden, int order,
                              __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const long long n = n_rows * hidden;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / hidden;
    const int c = (int)(i - r * hidden);
    const float v = x[i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    __nv_bfloat16* o = out + r * 3 * hidden + c;
    o[0] = hi;
    o[hidden] = order ? lo : hi;
    o[2 * hidden] = order ? hi : lo;
  }
}

// out[r][c] = in[r][a H + c] + in[r][b H + c] for in [n_rows][3H] (the gradient blocks of the
// fp32-faithful path that carry the hi and lo parts of the same operand).
__global__ void fold2_kernel(const float* __restrict__ in, long long n_rows, int hidden, int a, int b,
                             float* __restrict__ out) {
  pdl_enter();
  const long long n = n_rows * hidden;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / hidden;
    const int c = (int)(i - r * hidden);
    const float* row = in + r * 3 * hidden;
    out[i] = row[a * hidden + c] + row[b * hidden + c];
  }
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, long long n) {
  pdl_enter();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = i; j < n; j += stride) out[j] = __float2bfloat16_rn(in[j]);
}

// out = in * s with s = *g (1 when g is null): the autograd backward's scaling of a saved fp32
// gradient by the upstream gradient, written as bf16 (out_bf16) or fp32, in one pass.  n4 = n / 4
// float4 groups (pointers 16-byte aligned), then the n % 4 tail.
__global__ void scale_cast_kernel(const float* __restrict__ in, const float* __restrict__ g, long long n,
                                  void* __restrict__ out, int out_bf16) {
  pdl_enter();
  const float sc = g ? *g : 1.0f;
  const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long n4 = n >> 2;
  const float4* in4 = reinterpret_cast<const float4*>(in);
  for (long long j = i0; j < n4; j += stride) {
    const float4 v = in4[j];
    if (out_bf16) {
      uint2 o;
      o.x = pack_bf16x2(v.x * sc, v.y * sc);
      o.y = pack_bf16x2(v.z * sc, v.w * sc);
      reinterpret_cast<uint2*>(out)[j] = o;
    } else {
      reinterpret_cast<float4*>(out)[j] = make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc);
    }
  }
  for (long long j = 4 * n4 + i0; j < n; j += stride) {
    if (out_bf16) reinterpret_cast<__nv_bfloat16*>(out)[j] = __float2bfloat16_rn(in[j] * sc);
    else reinterpret_cast<float*>(out)[j] = in[j] * sc;
  }
}

}  // namespace klg
