// Block-diffusion attention, forward (inference), sm_100a.
//
// The reference's diffusion heads attend, for a query at diffusion position q of block
// q / K, to the AR key/value cache up to the query's causal limit (kv <= limit[b, q]) and to
// the K keys of their own block, bidirectionally (model.py:64-96 block mask + model.py:
// 435-446 score_mod, through flex_attention with GQA, model.py:45-58; the Triton version,
// triton_kernels.py:18-83, is marked broken).  Scores are scaled by 1 / sqrt(D).
//
// One CTA takes a unit (batch b, KV head, group of hg query heads sharing it, block) and a
// split of the AR key range.  Its queries -- hg heads x K positions <= 128 rows, zero rows
// after -- stay in shared memory; key tiles (128 AR keys, or the block's own K keys) stream
// through a TMA ring.  Per tile: S = Q K^T (tcgen05, M = 128, N = keys, K = 64) into the TMEM
// buffer of the tile's parity; the softmax warp group of that parity (four warps, one TMEM
// lane = one row per thread) takes the masked online max / sum in log2 units and writes
// P = 2^(s - m) as bf16 into its 128-byte-swizzled K-major shared tile; O_tile = P V
// (M = 128, N = 64, K = keys; V read MN-major) accumulates in the parity's TMEM O buffer
// (the group rescales that buffer in place on the rare tiles where a row's reference max
// moves, and reads it once at the end).  The MMA warp issues S one tile ahead,
// so the two groups (two warps per SM sub-partition) work on consecutive tiles at once;
// at the end the odd group's (m, l, O) is merged into the even group's through shared
// memory.  With one split the CTA writes bf16 O and the natural-log log-sum-exp itself.
// With several (decode: few units, the AR range split over up to 8 CTAs), the splits of a
// unit form one thread-block cluster: each CTA leaves its rows' (O, m, l) record in its own
// shared memory, and after a cluster barrier every CTA combines a share of the rows from all
// the records through distributed shared memory and writes them.
#pragma once
#include "klg_kernels.cuh"

namespace klg {

constexpr int ATT_D = 64;                              // head dimension
constexpr int ATT_BN = 128;                            // AR keys per tile
constexpr int ATT_STAGES = 3;
constexpr int ATT_TILE_BYTES = ATT_BN * ATT_D * 2;     // K or V tile, 16 KB
constexpr int ATT_Q_BYTES = 128 * ATT_D * 2;           // 16 KB
constexpr int ATT_P_BYTES = 128 * ATT_BN * 2;          // two 64-key K-major sub-tiles, 32 KB (per parity)
constexpr int ATT_X_BYTES = 128 * (ATT_D + 2) * 4;     // odd group's (O, m, l) handed to the even group
constexpr int ATT_THREADS = 320;                       // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
constexpr int ATT_SMEM = 1024 + ATT_Q_BYTES + 2 * ATT_P_BYTES + ATT_STAGES * 2 * ATT_TILE_BYTES + ATT_X_BYTES + 256;
constexpr int ATT_TMEM_COLS = 512;                     // S: 2 x 128 columns; O tiles: 2 x 64 at 256
constexpr int ATT_O_COL = 256;

struct AttnArgs {
  const int* limits;   // [B, Ld] causal limit per query position (AR keys 0..limit)
  __nv_bfloat16* out;  // O [B, H, Ld, 64]
  float* lse;          // [B, H, Ld] natural log, or null
  int B, H, Hkv, Ld, K, ar_len;
  int ng, hg, n_hg, nb;   // query heads per KV head, per unit; head groups; blocks
  int n_units, splits, tps;   // splits = cluster size (<= 8); tps: AR tiles per split
  float sl2;                  // scale * log2(e)
  int stall_split;            // test hook: the CTA of this split issues no key/value loads (-1: none)
};

// Units are numbered with the blocks of a sequence in reverse: later blocks see longer AR
// prefixes (their anchors come later), so CTAs start longest-first and the short units fill
// the tail of the grid.
__device__ __forceinline__ void attn_unit(const AttnArgs& a, int u, int& b, int& hkv, int& hgi, int& blk) {
  blk = a.nb - 1 - u % a.nb;
  int r = u / a.nb;
  hgi = r % a.n_hg;
  r /= a.n_hg;
  hkv = r % a.Hkv;
  b = r / a.Hkv;
}

// One 32-key chunk c of a row of S (raw fp32 bits): P = 2^(s sl2 - ref) for the visible keys
// (key <= kmax; all of them when `open`), written as bf16 into the row's swizzled P tile;
// folds the chunk's max (scaled) and sum into tmax / sum.
__device__ __forceinline__ void attn_p_chunk(const uint32_t (&v)[32], int c, int nk, int kmax, bool open, float sl2,
                                             float ref, uint32_t prow, int r, float& tmax, float& sum) {
  uint32_t pk[16];   // P as bf16 pairs
  float t0 = -INFINITY, t1 = -INFINITY;
  uint64_t ss = 0;   // packed (s0, s1) = (0.f, 0.f): the even and odd keys' sums
  const uint64_t sl2x2 = f2_pack(sl2, sl2), nref = f2_pack(-ref, -ref);
  if (open) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float x0 = __uint_as_float(v[j]), x1 = __uint_as_float(v[j + 1]);
      t0 = fmaxf(t0, x0);
      t1 = fmaxf(t1, x1);
      float a0, a1;
      f2_unpack(f2_fma(f2_pack(x0, x1), sl2x2, nref), a0, a1);
      const float p0 = ex2(a0), p1 = ex2(a1);
      ss = f2_add(ss, f2_pack(p0, p1));
      pk[j >> 1] = pack_bf16x2(p0, p1);
    }
    tmax = fmaxf(tmax, fmaxf(t0, t1) * sl2);   // scale > 0 commutes with max
  } else {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      float x0, x1;
      f2_unpack(f2_mul(f2_pack(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), sl2x2), x0, x1);
      x0 = c * 32 + j <= kmax ? x0 : -INFINITY;
      x1 = c * 32 + j + 1 <= kmax ? x1 : -INFINITY;
      t0 = fmaxf(t0, x0);
      t1 = fmaxf(t1, x1);
      float a0, a1;
      f2_unpack(f2_add(f2_pack(x0, x1), nref), a0, a1);
      const float p0 = ex2(a0), p1 = ex2(a1);
      ss = f2_add(ss, f2_pack(p0, p1));
      pk[j >> 1] = pack_bf16x2(p0, p1);
    }
    tmax = fmaxf(tmax, fmaxf(t0, t1));
  }
  float s0, s1;
  f2_unpack(ss, s0, s1);
  sum += s0 + s1;
#pragma unroll
  for (int q8 = 0; q8 < 4; ++q8) {
    const int chunk = c * 4 + q8;   // 8 keys = 16 bytes; 8 chunks per 64-key sub-tile row
    if (chunk * 8 < nk) {
      const uint32_t addr = prow + (uint32_t)(chunk >> 3) * 16384u + (uint32_t)(((chunk & 7) ^ (r & 7)) << 4);
      st_shared_v4(addr, pk[4 * q8], pk[4 * q8 + 1], pk[4 * q8 + 2], pk[4 * q8 + 3]);
    }
  }
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
block_attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_ks,
                  const __grid_constant__ CUtensorMap map_vs, const __grid_constant__ CUtensorMap map_ka,
                  const __grid_constant__ CUtensorMap map_va, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int s_maxlim;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t q_s = smem_u32(smem);
  const uint32_t p_s = q_s + ATT_Q_BYTES;                  // [2] P tiles, one per parity
  const uint32_t st_s = p_s + 2 * ATT_P_BYTES;   // stage j: K tile at st_s + 2j * TILE, V tile right after
  float* xch = reinterpret_cast<float*>(smem + ATT_Q_BYTES + 2 * ATT_P_BYTES + ATT_STAGES * 2 * ATT_TILE_BYTES);
  const uint32_t bar0 = st_s + ATT_STAGES * 2 * ATT_TILE_BYTES + ATT_X_BYTES;
  const uint32_t full0 = bar0;                        // [STAGES] TMA bytes of K + V
  const uint32_t empty0 = bar0 + 8u * ATT_STAGES;     // [STAGES] P V of the stage retired
  const uint32_t qbar = bar0 + 16u * ATT_STAGES;      // queries landed
  const uint32_t sfull0 = qbar + 8u;                  // [2] S tile in TMEM (per parity)
  const uint32_t sempty0 = sfull0 + 16u;              // [2] the parity's softmax warps read it
  const uint32_t pfull0 = sempty0 + 16u;              // [2] P written to shared memory
  const uint32_t ofull0 = pfull0 + 16u;               // [2] the parity's latest P V retired
  const uint32_t done_bar = ofull0 + 16u;             // every MMA this CTA issued retired
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int u = blockIdx.x / a.splits;
  const int sp = blockIdx.x - u * a.splits;
  int b, hkv, hgi, blk;
  attn_unit(a, u, b, hkv, hgi, blk);
  const int rows = a.hg * a.K;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    s_maxlim = -1;
    for (int s = 0; s < ATT_STAGES; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    mbar_init(qbar, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(sfull0 + 8u * s, 1);
      mbar_init(sempty0 + 8u * s, 4);
      mbar_init(pfull0 + 8u * s, 4);
      mbar_init(ofull0 + 8u * s, 1);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch(&map_q);
    tma_prefetch(&map_ks);
    tma_prefetch(&map_vs);
    tma_prefetch(&map_ka);
    tma_prefetch(&map_va);
  }
  // query rows past the unit's rows: zeros (their S / P rows are formed and never read)
  for (int i = threadIdx.x; i < (128 - rows) * 8; i += blockDim.x) st_shared_v4(q_s + rows * 128 + i * 16, 0, 0, 0, 0);
  fence_async_shared();
  if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), ATT_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_enter();   // inputs of this launch are complete from here on
  if (threadIdx.x < a.K) atomicMax(&s_maxlim, a.limits[(size_t)b * a.Ld + blk * a.K + threadIdx.x]);
  __syncthreads();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;
  const int maxlim = min(s_maxlim, a.ar_len - 1);
  const int n_ar = maxlim < 0 ? 0 : maxlim / ATT_BN + 1;   // AR tiles holding keys 0..maxlim
  const int t0 = sp * a.tps;
  const int n_my = max(0, min(t0 + a.tps, n_ar) - t0);
  const int ntiles = n_my + (sp == a.splits - 1 ? 1 : 0);   // the last split also takes the block's own keys

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (whole warp)
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    if (elect_one()) {
      mbar_arrive_expect_tx(qbar, (uint32_t)rows * 128u);
      for (int i = 0; i < a.hg; ++i) {
        const int h = hkv * a.ng + hgi * a.hg + i;
        tma_load_2d(q_s + i * a.K * 128, &map_q, qbar, 0, (b * a.H + h) * a.Ld + blk * a.K);
      }
    }
    __syncwarp();
    // (test hook) a stalled split loads no tiles: its MMA warp's first operand wait runs out its
    // bound, and the CTA still reaches both cluster barriers below
    const int n_load = sp == a.stall_split ? 0 : ntiles;
    for (int i = 0; i < n_load; ++i) {
      if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) break;
      if (elect_one()) {
        const uint32_t ks = st_s + stage * 2 * ATT_TILE_BYTES;
        const uint32_t fb = full0 + 8u * stage;
        if (i < n_my) {
          mbar_arrive_expect_tx(fb, 2 * ATT_TILE_BYTES);
          tma_load_3d(ks, &map_ka, fb, 0, (t0 + i) * ATT_BN, b * a.Hkv + hkv);
          tma_load_3d(ks + ATT_TILE_BYTES, &map_va, fb, 0, (t0 + i) * ATT_BN, b * a.Hkv + hkv);
        } else {
          mbar_arrive_expect_tx(fb, (uint32_t)(2 * a.K * 128));
          const int row = (b * a.Hkv + hkv) * a.Ld + blk * a.K;
          tma_load_2d(ks, &map_ks, fb, 0, row);
          tma_load_2d(ks + ATT_TILE_BYTES, &map_vs, fb, 0, row);
        }
      }
      __syncwarp();
      ++issued;
      if (++stage == ATT_STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (lane == 0) {
      drain_loads<ATT_STAGES>(full0, stage, phase, issued);
      mbar_wait_drain(qbar, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp)
    // S of tile i + 1 is issued before P V of tile i, so both softmax groups have work.
    bool ok = warp_wait(qbar, 0, abort_p, KLG_STATUS_TIMEOUT_MMA);
    tc_fence_after();
    auto issue_s = [&](int i) -> bool {   // S_i = Q K_i^T into the parity's S buffer
      const int stage = i % ATT_STAGES;
      const uint32_t phase = (uint32_t)(i / ATT_STAGES) & 1u;
      const int par = i & 1;
      if (!warp_wait(full0 + 8u * stage, phase, abort_p, KLG_STATUS_TIMEOUT_MMA)) return false;
      if (!warp_wait(sempty0 + 8u * par, ((uint32_t)(i >> 1) & 1u) ^ 1u, abort_p, KLG_STATUS_TIMEOUT_MMA)) return false;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t idesc = make_idesc_bf16(128, i < n_my ? ATT_BN : a.K, false, false);
        const uint32_t ks = st_s + stage * 2 * ATT_TILE_BYTES;
#pragma unroll
        for (int k = 0; k < ATT_D / 16; ++k)
          mma_bf16(tmem + par * ATT_BN, desc_kmajor(q_s, k), desc_kmajor(ks, k), idesc, k != 0);
        mma_commit(sfull0 + 8u * par);
      }
      __syncwarp();
      return true;
    };
    if (ok && ntiles > 0) ok = issue_s(0);
    for (int i = 0; ok && i < ntiles; ++i) {
      if (i + 1 < ntiles && !(ok = issue_s(i + 1))) break;
      const int par = i & 1;
      const int stage = i % ATT_STAGES;
      const int nk = i < n_my ? ATT_BN : a.K;
      if (!warp_wait(pfull0 + 8u * par, (uint32_t)(i >> 1) & 1u, abort_p, KLG_STATUS_TIMEOUT_MMA)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t idesc = make_idesc_bf16(128, ATT_D, false, true);
        const uint32_t vs = st_s + stage * 2 * ATT_TILE_BYTES + ATT_TILE_BYTES;
        const uint32_t pp = p_s + par * ATT_P_BYTES;
        for (int k = 0; k < nk / 16; ++k)
          mma_bf16(tmem + ATT_O_COL + par * ATT_D, desc_kmajor(pp + (k >> 2) * 16384, k & 3), desc_mnmajor(vs, k),
                   idesc, (k != 0 || i >= 2) ? 1u : 0u);   // the parity's first tile starts O
        mma_commit(ofull0 + 8u * par);
        mma_commit(empty0 + 8u * stage);
      }
      __syncwarp();
    }
    // every MMA issued above has retired before TMEM is freed, also when a wait gave up
    // with an S tile still in flight that no softmax warp will read
    if (elect_one()) mma_commit(done_bar);
    __syncwarp();
    mbar_wait_drain(done_bar, 0);
  } else {
    // ------------------------------------------------------------ softmax warps (one row per thread)
    const int q4 = warp & 3;   // TMEM lane quarter of this warp
    const int par = (warp - 2) >> 2;   // tiles of this parity
    const int r = q4 * 32 + lane;
    const int pos = r % a.K;
    const int lim = r < rows ? min(max(a.limits[(size_t)b * a.Ld + blk * a.K + pos], -1), a.ar_len - 1) : -1;
    const uint32_t lrow = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t prow = p_s + par * ATT_P_BYTES + (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u;
    float m = NEG_BIG, l = 0.f;
    bool ok = true;
    int n_pv = 0;   // P V products this group handed to the MMA warp
    for (int i = par; ok && i < ntiles; i += 2) {
      const bool self = i >= n_my;
      const int nk = self ? a.K : ATT_BN;
      const int kmax = self ? a.K - 1 : lim - (t0 + i) * ATT_BN;   // last visible key of the tile
      const int sb = par;
      const uint32_t jph = (uint32_t)(i >> 1) & 1u;   // this parity's use count of its S buffer
      if (!mbar_wait(sfull0 + 8u * sb, jph, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // P of this parity's previous tile is still an MMA operand until its P V completes
      if (n_pv > 0 && !mbar_wait(ofull0 + 8u * sb, (uint32_t)(n_pv - 1) & 1u, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      const int nch = (nk + 31) >> 5;
      // every key of the tile visible to all 32 rows of the warp: no per-key mask
      const bool open = __all_sync(0xffffffffu, kmax >= nk - 1) && (nk & 31) == 0;
      // One pass over S writes P = 2^(s - ref) for the reference max `ref` and returns the
      // tile's max and sum.  (Double-buffering the TMEM loads needs 64 more registers than the
      // 168 a thread can have with ten warps -- three per SM sub-partition -- and spills.)
      auto p_pass = [&](float ref, float& tmax, float& sum) {
        tmax = -INFINITY;
        sum = 0.f;
        for (int c = 0; c < nch; ++c) {
          uint32_t v[32];
          tmem_ld32_raw(lrow + sb * ATT_BN + c * 32, v);
          tmem_wait_ld_regs(v);
          attn_p_chunk(v, c, nk, kmax, open, a.sl2, ref, prow, r, tmax, sum);
        }
      };
      // P against the running max; only when a row's tile max exceeds it by more than 2^10
      // (always on a row's first visible tile) is the tile redone against the new max.  l and
      // O use the same reference either way, so the result is exact; P stays <= 2^10.
      float tmax, sum;
      p_pass(m, tmax, sum);
      float mn = m;
      if (__any_sync(0xffffffffu, tmax > m + 10.f)) {
        mn = fmaxf(m, tmax);
        p_pass(mn, tmax, sum);
      }
      const float alpha = ex2(m - mn);
      l = fmaf(l, alpha, sum);
      m = mn;
      // a moved reference: rescale the O accumulated so far (its last P V completed above)
      if (n_pv > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v[32];
          tmem_ld32_raw(lrow + ATT_O_COL + par * ATT_D + h * 32, v);
          tmem_wait_ld_regs(v);
          float w[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) w[j] = __uint_as_float(v[j]) * alpha;
          tmem_st32(lrow + ATT_O_COL + par * ATT_D + h * 32, w);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(sempty0 + 8u * sb);
        mbar_arrive(pfull0 + 8u * sb);
      }
      ++n_pv;
    }
    // the group's O: its last P V retired (bounded wait even after an abort, so no MMA is in
    // flight when TMEM is freed)
    float o[ATT_D];
    bool have = false;
    if (n_pv > 0 && (ok ? mbar_wait(ofull0 + 8u * par, (uint32_t)(n_pv - 1) & 1u, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)
                        : mbar_wait_drain(ofull0 + 8u * par, (uint32_t)(n_pv - 1) & 1u))) {
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32_raw(lrow + ATT_O_COL + par * ATT_D, v0);
      tmem_ld32_raw(lrow + ATT_O_COL + par * ATT_D + 32, v1);
      tmem_wait_ld_regs(v0, v1);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        o[j] = __uint_as_float(v0[j]);
        o[32 + j] = __uint_as_float(v1[j]);
      }
      have = ok;
    }
    if (!have) {   // no tile, or a group that gave up: contributes nothing
      m = NEG_BIG;
      l = 0.f;
#pragma unroll
      for (int j = 0; j < ATT_D; ++j) o[j] = 0.f;
    }
    // the odd group hands its state to the even group through shared memory
    float* x = xch + r * (ATT_D + 2);
    if (par == 1) {
#pragma unroll
      for (int j = 0; j < ATT_D; ++j) x[j] = o[j];
      x[ATT_D] = m;
      x[ATT_D + 1] = l;
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");   // the eight softmax warps
    if (par == 0) {
      const float m1 = x[ATT_D];
      const float mm = fmaxf(m, m1);
      const float w0 = ex2(m - mm), w1 = ex2(m1 - mm);
      l = l * w0 + x[ATT_D + 1] * w1;
      m = mm;
#pragma unroll
      for (int j = 0; j < ATT_D; ++j) o[j] = o[j] * w0 + x[j] * w1;
      if (a.splits == 1) {
        // the whole key range is here: normalise and write the output row directly
        if (r < rows) {
          const int h = hkv * a.ng + hgi * a.hg + r / a.K;
          const size_t row = ((size_t)b * a.H + h) * a.Ld + blk * a.K + pos;
          const float inv = l > 0.f ? 1.0f / l : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(a.out + row * ATT_D);
#pragma unroll
          for (int j = 0; j < ATT_D / 8; ++j)
            dst[j] = make_uint4(pack_bf16x2(o[8 * j] * inv, o[8 * j + 1] * inv),
                                pack_bf16x2(o[8 * j + 2] * inv, o[8 * j + 3] * inv),
                                pack_bf16x2(o[8 * j + 4] * inv, o[8 * j + 5] * inv),
                                pack_bf16x2(o[8 * j + 6] * inv, o[8 * j + 7] * inv));
          if (a.lse) a.lse[row] = (m + __log2f(l)) * 0.69314718055994530942f;
        }
      } else {
        // this split's record of the row, in place of the odd group's state it just read
        // (same thread, same row); also written when the split had no tiles
#pragma unroll
        for (int j = 0; j < ATT_D; ++j) x[j] = o[j];
        x[ATT_D] = m;
        x[ATT_D + 1] = l;
      }
    }
  }
  // Every thread of every CTA of the cluster must reach both cluster barriers: they have no
  // time bound.  Nothing above returns early -- each role leaves its loop on a bounded wait
  // that gave up (or on the CTA's abort flag) and falls through to here -- and any early exit
  // added above would leave the other splits of the unit waiting here for good.
  if (a.splits > 1) {
    cluster_sync();   // every split's records of the unit are in its CTA's shared memory
    const uint32_t rank = cluster_rank();
    const uint32_t xbase = smem_u32(xch);
    // rows rank, rank + splits, ...: one warp per row, lane j reads split j's (m, l) and then
    // two head-dimension columns of every split's O
    for (int rr = (int)rank + a.splits * warp; rr < rows; rr += a.splits * (ATT_THREADS / 32)) {
      const uint32_t rec = xbase + (uint32_t)(rr * (ATT_D + 2)) * 4u;
      float mj = NEG_BIG, lj = 0.f;
      if (lane < a.splits) {
        const uint32_t peer = mapa_shared(rec, (uint32_t)lane);
        mj = ld_shared_cluster_f32(peer + ATT_D * 4);
        lj = ld_shared_cluster_f32(peer + (ATT_D + 1) * 4);
      }
      float M = mj;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      const float w = lane < a.splits ? ex2(mj - M) : 0.f;
      float L = lj * w;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      float o0 = 0.f, o1 = 0.f;
      for (int sp2 = 0; sp2 < a.splits; ++sp2) {
        const float wp = __shfl_sync(0xffffffffu, w, sp2);
        const uint32_t peer = mapa_shared(rec + (uint32_t)(2 * lane) * 4u, (uint32_t)sp2);
        o0 = fmaf(ld_shared_cluster_f32(peer), wp, o0);
        o1 = fmaf(ld_shared_cluster_f32(peer + 4), wp, o1);
      }
      const int h = hkv * a.ng + hgi * a.hg + rr / a.K;
      const size_t row = ((size_t)b * a.H + h) * a.Ld + blk * a.K + rr % a.K;
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      reinterpret_cast<uint32_t*>(a.out + row * ATT_D)[lane] = pack_bf16x2(o0 * inv, o1 * inv);
      if (a.lse && lane == 0) a.lse[row] = (M + __log2f(L)) * 0.69314718055994530942f;
    }
    cluster_sync();   // no CTA leaves while a peer may still read its records
  }
  tc_fence_before();
  __syncthreads();   // every MMA retired (the softmax warps consumed the last O tile) before TMEM is freed
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, ATT_TMEM_COLS);
}


// =====================================================================================
// Backward (training the diffusion heads): dQ, and dK / dV of the block's own keys.
//
// Per unit (batch b, KV head, group of hg query heads sharing it, block) one CTA walks the
// key tiles of the forward -- the AR tiles the block's limits reach, then the block's own K
// keys -- with the forward's row log-sum-exps: S = Q K^T and dP = dO V^T (tcgen05, TMEM),
// then softmax warps (one query row per thread) form P = 2^(s sl2 - lse2) on the visible keys
// and dS = P (dP - D), D = rowsum(dO O), as bf16 tiles in shared memory; the MMA warp
// accumulates dQ += dS K in TMEM across tiles and, on the block's own tile, dV = P^T dO and
// dK = dS^T Q (the unit's rows cover every query head of the group, so these sum over the
// heads sharing the KV head).  The AR cache gets no gradient: it comes from the frozen
// backbone (the reference's Triton backward, triton_kernels.py:73-141 / 161-172, returns
// none for it either).  dq and the self keys' dk / dv are fp32; with more than one head group
// per KV head the units add into dk / dv (the host zeroes them first).
// =====================================================================================
constexpr int ATB_STAGES = 2;
constexpr int ATB_THREADS = 320;                       // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
constexpr int ATB_SMEM = 1024 + 2 * ATT_Q_BYTES + 2 * ATT_P_BYTES + ATB_STAGES * 2 * ATT_TILE_BYTES + 256;
constexpr int ATB_S_COL = 0, ATB_DP_COL = 128, ATB_DQ_COL = 256, ATB_DV_COL = 320, ATB_DK_COL = 384;

struct AttnBwdArgs {
  const int* limits;          // [B, Ld]
  const __nv_bfloat16* out;   // forward output O [B, H, Ld, 64]
  const __nv_bfloat16* dout;  // upstream gradient dO [B, H, Ld, 64]
  const float* lse;           // forward log-sum-exp [B, H, Ld], natural log
  float* dq;                  // [B, H, Ld, 64]
  float* dk;                  // [B, Hkv, Ld, 64] (self keys)
  float* dv;                  // [B, Hkv, Ld, 64]
  int B, H, Hkv, Ld, K, ar_len;
  int ng, hg, n_hg, nb, n_units;
  float scale;                // softmax scale (scores = scale q k)
  float sl2;                  // scale * log2(e)
  int accumulate_kv;          // 1: add into dk / dv (several head groups per KV head)
};

__device__ __forceinline__ void attn_bwd_unit(const AttnBwdArgs& a, int u, int& b, int& hkv, int& hgi, int& blk) {
  blk = a.nb - 1 - u % a.nb;
  int r = u / a.nb;
  hgi = r % a.n_hg;
  r /= a.n_hg;
  hkv = r % a.Hkv;
  b = r / a.Hkv;
}

// Writes 32 bf16 (one row r, keys c32 * 32 .. + 31 of a 128-key tile) into a tile stored as
// two 64-key K-major sub-tiles with the 128-byte swizzle (the forward's P layout).
__device__ __forceinline__ void atb_store_row32(uint32_t tile, int r, int c32, const uint32_t (&pk)[16]) {
  const uint32_t rowb = tile + (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u;
#pragma unroll
  for (int q8 = 0; q8 < 4; ++q8) {
    const int chunk = c32 * 4 + q8;   // 8 keys = 16 bytes
    st_shared_v4(rowb + (uint32_t)(chunk >> 3) * 16384u + (uint32_t)(((chunk & 7) ^ (r & 7)) << 4), pk[4 * q8],
                 pk[4 * q8 + 1], pk[4 * q8 + 2], pk[4 * q8 + 3]);
  }
}

__global__ void __launch_bounds__(ATB_THREADS, 1)
block_attn_bwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_do,
                      const __grid_constant__ CUtensorMap map_ks, const __grid_constant__ CUtensorMap map_vs,
                      const __grid_constant__ CUtensorMap map_ka, const __grid_constant__ CUtensorMap map_va,
                      const AttnBwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int s_maxlim;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t q_s = smem_u32(smem);
  const uint32_t do_s = q_s + ATT_Q_BYTES;
  const uint32_t p_s = do_s + ATT_Q_BYTES;              // P tile (self tile only), two 64-key sub-tiles
  const uint32_t ds_s = p_s + ATT_P_BYTES;              // dS tile
  const uint32_t st_s = ds_s + ATT_P_BYTES;             // stage j: K tile, then V tile
  const uint32_t bar0 = st_s + ATB_STAGES * 2 * ATT_TILE_BYTES;
  const uint32_t full0 = bar0;                          // [STAGES] K + V bytes landed
  const uint32_t empty0 = bar0 + 8u * ATB_STAGES;       // [STAGES] the stage's MMAs retired
  const uint32_t qbar = bar0 + 16u * ATB_STAGES;        // Q and dO landed
  const uint32_t sfull = qbar + 8u;                     // S and dP of the current tile in TMEM
  const uint32_t pfull = sfull + 8u;                    // the softmax warps wrote P / dS and read S / dP
  const uint32_t dsfree = pfull + 8u;                   // the MMAs reading P / dS retired
  const uint32_t done_bar = dsfree + 8u;                // every MMA of the CTA retired
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int b, hkv, hgi, blk;
  attn_bwd_unit(a, blockIdx.x, b, hkv, hgi, blk);
  const int rows = a.hg * a.K;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    s_maxlim = -1;
    for (int s = 0; s < ATB_STAGES; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    mbar_init(qbar, 1);
    mbar_init(sfull, 1);
    mbar_init(pfull, 8);
    mbar_init(dsfree, 1);
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch(&map_q);
    tma_prefetch(&map_do);
    tma_prefetch(&map_ks);
    tma_prefetch(&map_vs);
    tma_prefetch(&map_ka);
    tma_prefetch(&map_va);
  }
  // rows past the unit's: zero queries and upstream gradients (their P / dS rows are zero too)
  for (int i = threadIdx.x; i < (128 - rows) * 8; i += blockDim.x) {
    st_shared_v4(q_s + rows * 128 + i * 16, 0, 0, 0, 0);
    st_shared_v4(do_s + rows * 128 + i * 16, 0, 0, 0, 0);
  }
  fence_async_shared();
  if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), ATT_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_enter();   // inputs of this launch are complete from here on
  if (threadIdx.x < a.K) atomicMax(&s_maxlim, a.limits[(size_t)b * a.Ld + blk * a.K + threadIdx.x]);
  __syncthreads();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;
  const int maxlim = min(s_maxlim, a.ar_len - 1);
  const int n_ar = maxlim < 0 ? 0 : maxlim / ATT_BN + 1;   // AR tiles holding keys 0..maxlim
  const int ntiles = n_ar + 1;                             // + the block's own keys

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (whole warp)
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    if (elect_one()) {
      mbar_arrive_expect_tx(qbar, 2u * (uint32_t)rows * 128u);
      for (int i = 0; i < a.hg; ++i) {
        const int h = hkv * a.ng + hgi * a.hg + i;
        const int grow = (b * a.H + h) * a.Ld + blk * a.K;
        tma_load_2d(q_s + i * a.K * 128, &map_q, qbar, 0, grow);
        tma_load_2d(do_s + i * a.K * 128, &map_do, qbar, 0, grow);
      }
    }
    __syncwarp();
    for (int i = 0; i < ntiles; ++i) {
      if (!warp_wait(empty0 + 8u * stage, phase ^ 1, abort_p, KLG_STATUS_TIMEOUT_PRODUCER)) break;
      if (elect_one()) {
        const uint32_t ks = st_s + stage * 2 * ATT_TILE_BYTES;
        const uint32_t fb = full0 + 8u * stage;
        if (i < n_ar) {
          mbar_arrive_expect_tx(fb, 2 * ATT_TILE_BYTES);
          tma_load_3d(ks, &map_ka, fb, 0, i * ATT_BN, b * a.Hkv + hkv);
          tma_load_3d(ks + ATT_TILE_BYTES, &map_va, fb, 0, i * ATT_BN, b * a.Hkv + hkv);
        } else {
          mbar_arrive_expect_tx(fb, (uint32_t)(2 * a.K * 128));
          const int row = (b * a.Hkv + hkv) * a.Ld + blk * a.K;
          tma_load_2d(ks, &map_ks, fb, 0, row);
          tma_load_2d(ks + ATT_TILE_BYTES, &map_vs, fb, 0, row);
        }
      }
      __syncwarp();
      ++issued;
      if (++stage == ATB_STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (lane == 0) {
      drain_loads<ATB_STAGES>(full0, stage, phase, issued);
      mbar_wait_drain(qbar, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp)
    bool ok = warp_wait(qbar, 0, abort_p, KLG_STATUS_TIMEOUT_MMA);
    tc_fence_after();
    auto issue_s_dp = [&](int i) -> bool {   // S_i = Q K_i^T and dP_i = dO V_i^T
      const int stage = i % ATB_STAGES;
      if (!warp_wait(full0 + 8u * stage, (uint32_t)(i / ATB_STAGES) & 1u, abort_p, KLG_STATUS_TIMEOUT_MMA)) return false;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t idesc = make_idesc_bf16(128, i < n_ar ? ATT_BN : a.K, false, false);
        const uint32_t ks = st_s + stage * 2 * ATT_TILE_BYTES;
#pragma unroll
        for (int k = 0; k < ATT_D / 16; ++k) {
          mma_bf16(tmem + ATB_S_COL, desc_kmajor(q_s, k), desc_kmajor(ks, k), idesc, k != 0);
          mma_bf16(tmem + ATB_DP_COL, desc_kmajor(do_s, k), desc_kmajor(ks + ATT_TILE_BYTES, k), idesc, k != 0);
        }
        mma_commit(sfull);
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = issue_s_dp(0);
    for (int i = 0; ok && i < ntiles; ++i) {
      const int stage = i % ATB_STAGES;
      const bool self = i == n_ar;
      const int nk = self ? a.K : ATT_BN;
      // the softmax warps wrote P_i / dS_i and are done with S_i / dP_i in TMEM
      if (!warp_wait(pfull, (uint32_t)i & 1u, abort_p, KLG_STATUS_TIMEOUT_MMA)) { ok = false; break; }
      tc_fence_after();
      if (elect_one()) {
        const uint32_t ks = st_s + stage * 2 * ATT_TILE_BYTES;
        const uint32_t idesc_q = make_idesc_bf16(128, ATT_D, false, true);
        for (int k = 0; k < nk / 16; ++k)   // dQ += dS K (K-major dS, K read MN-major)
          mma_bf16(tmem + ATB_DQ_COL, desc_kmajor(ds_s + (k >> 2) * 16384, k & 3), desc_mnmajor(ks, k), idesc_q,
                   (k != 0 || i != 0) ? 1u : 0u);
        if (self) {   // dV = P^T dO, dK = dS^T Q over the unit's 128 (padded) query rows
          const uint32_t idesc_t = make_idesc_bf16(128, ATT_D, true, true);
#pragma unroll
          for (int k = 0; k < 128 / 16; ++k) {
            mma_bf16(tmem + ATB_DV_COL, make_desc_sw128(p_s + 2048u * k, 16384u, 1024u), desc_mnmajor(do_s, k),
                     idesc_t, k != 0);
            mma_bf16(tmem + ATB_DK_COL, make_desc_sw128(ds_s + 2048u * k, 16384u, 1024u), desc_mnmajor(q_s, k),
                     idesc_t, k != 0);
          }
        }
        mma_commit(empty0 + 8u * stage);   // K_i / V_i free once these retire
        mma_commit(dsfree);                // P_i / dS_i free once these retire
      }
      __syncwarp();
      if (i + 1 < ntiles && !(ok = issue_s_dp(i + 1))) break;
    }
    if (elect_one()) mma_commit(done_bar);
    __syncwarp();
    mbar_wait_drain(done_bar, 0);
  } else {
    // ------------------------------------------------------------ softmax warps (one row per thread)
    const int q4 = warp & 3;
    const int hf = (warp - 2) >> 2;   // key half (64 keys) of each tile
    const int r = q4 * 32 + lane;
    const bool live = r < rows;
    const int h = hkv * a.ng + hgi * a.hg + (live ? r / a.K : 0);
    const int pos = r % a.K;
    const size_t grow = ((size_t)(b * a.H + h) * a.Ld + blk * a.K + pos);
    const int lim = live ? min(max(a.limits[(size_t)b * a.Ld + blk * a.K + pos], -1), a.ar_len - 1) : -1;
    const float lse2 = live ? a.lse[grow] * 1.4426950408889634f : 0.f;
    // D = rowsum(dO * O) of the forward output
    float D = 0.f;
    if (live) {
      const uint4* o4 = reinterpret_cast<const uint4*>(a.out + grow * ATT_D);
      const uint4* d4 = reinterpret_cast<const uint4*>(a.dout + grow * ATT_D);
#pragma unroll
      for (int j = 0; j < ATT_D / 8; ++j) {
        const uint4 ov = o4[j], dv = d4[j];
        const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          D = fmaf(__uint_as_float(ow[t] << 16), __uint_as_float(dw[t] << 16), D);
          D = fmaf(__uint_as_float(ow[t] & 0xFFFF0000u), __uint_as_float(dw[t] & 0xFFFF0000u), D);
        }
      }
    }
    const uint32_t lrow = tmem + ((uint32_t)(q4 * 32) << 16);
    bool ok = true;
    for (int i = 0; ok && i < ntiles; ++i) {
      const bool self = i == n_ar;
      if (!mbar_wait(sfull, (uint32_t)i & 1u, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
      // P / dS of the previous tile are still MMA operands until those MMAs retire
      if (i > 0 && !mbar_wait(dsfree, (uint32_t)(i - 1) & 1u, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int c32 = hf * 2 + c;                  // 32-key chunk of the 128-key tile
        uint32_t sv[32], pv[32];
        tmem_ld32_raw(lrow + ATB_S_COL + c32 * 32, sv);
        tmem_ld32_raw(lrow + ATB_DP_COL + c32 * 32, pv);
        tmem_wait_ld_regs(sv, pv);
        uint32_t pp[16], dd[16];
        const uint64_t sl2x2 = f2_pack(a.sl2, a.sl2), nlse = f2_pack(-lse2, -lse2), dd2 = f2_pack(D, D);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const int key0 = c32 * 32 + j;             // key index within the tile
          const bool v0 = live && (self ? key0 < a.K : i * ATT_BN + key0 <= lim);
          const bool v1 = live && (self ? key0 + 1 < a.K : i * ATT_BN + key0 + 1 <= lim);
          float e0, e1;   // packed fp32x2: the same roundings as the scalar form
          f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1])), sl2x2, nlse), e0, e1);
          const float p0 = v0 ? ex2(e0) : 0.f;
          const float p1 = v1 ? ex2(e1) : 0.f;
          const uint64_t p = f2_pack(p0, p1);
          float d0, d1;
          f2_unpack(f2_mul(p, f2_sub(f2_pack(__uint_as_float(pv[j]), __uint_as_float(pv[j + 1])), dd2)), d0, d1);
          pp[j / 2] = pack_bf16x2(p0, p1);
          dd[j / 2] = pack_bf16x2(d0, d1);
        }
        atb_store_row32(ds_s, r, c32, dd);
        if (self) atb_store_row32(p_s, r, c32, pp);
      }
      tc_fence_before();
      fence_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull);
    }
    // dQ (this warp's 32 of the 64 columns), and dK / dV of the block's own keys
    const bool fin = mbar_wait(done_bar, 0, abort_p, KLG_STATUS_TIMEOUT_EPILOGUE);
    tc_fence_after();
    if (fin && ok) {
      uint32_t v[32];
      tmem_ld32_raw(lrow + ATB_DQ_COL + hf * 32, v);
      tmem_wait_ld_regs(v);
      if (live) {
        float4* dst = reinterpret_cast<float4*>(a.dq + grow * ATT_D + hf * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          dst[j] = make_float4(__uint_as_float(v[4 * j]) * a.scale, __uint_as_float(v[4 * j + 1]) * a.scale,
                               __uint_as_float(v[4 * j + 2]) * a.scale, __uint_as_float(v[4 * j + 3]) * a.scale);
      }
      const int key = r;   // TMEM lane of dK / dV = the block's key index
      const size_t krow = ((size_t)(b * a.Hkv + hkv) * a.Ld + blk * a.K + key);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        tmem_ld32_raw(lrow + (t ? ATB_DK_COL : ATB_DV_COL) + hf * 32, v);
        tmem_wait_ld_regs(v);
        if (key < a.K) {
          float* dst = (t ? a.dk : a.dv) + krow * ATT_D + hf * 32;
          const float sc = t ? a.scale : 1.f;
          if (a.accumulate_kv) {
#pragma unroll
            for (int j = 0; j < 32; ++j) atomicAdd(dst + j, __uint_as_float(v[j]) * sc);
          } else {
            float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              d4[j] = make_float4(__uint_as_float(v[4 * j]) * sc, __uint_as_float(v[4 * j + 1]) * sc,
                                  __uint_as_float(v[4 * j + 2]) * sc, __uint_as_float(v[4 * j + 3]) * sc);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();   // every MMA retired (done_bar) before TMEM is freed
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, ATT_TMEM_COLS);
}

}  // namespace klg
