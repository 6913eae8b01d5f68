// Cross-rank dW exchange for row-sharded training over NVLink peer memory, sm_100a.
//
// With the rows sharded over `world` ranks every rank computes a partial dW [V, H] for its own
// rows, and the data-parallel step needs their sum on every rank.  Instead of an all-reduce
// after the step, the dW GEMM's epilogue (gemm_pair_kernel with XrArgs) stores each 32-row
// block of its partial straight into the inbox of the block's owner -- block b belongs to rank
// b % world -- while the pass-2 GEMMs run (plain 16-byte peer stores, no atomics; a K-split
// tile's two halves go to two slots).  Two small kernels finish the step:
//
//   xr_reduce_kernel  signals "pushed, epoch e" to every rank, waits for every rank's signal,
//                     and sums its own blocks over (rank, K half) in a fixed order into its
//                     `final` rows;
//   xr_wait_kernel    (one block) signals "reduced, epoch e" and waits for every rank's; then
//                     the copy engines fetch each owner's `final` rows over NVLink into their
//                     32-row blocks of the local dW (one strided cudaMemcpy2DAsync per owner,
//                     no SMs).
//
// The ordering also holds across steps: a rank pushes step e + 1 only after its copies of
// step e, which come after every rank's reduce of step e; a rank's reduce of step e + 1
// overwrites its `final` rows only after every rank has pushed step e + 1, i.e. after every
// rank's copies of step e -- so no inbox or final row is overwritten while another rank
// still reads it.  The fixed summation order makes dW the
// same on every rank and the same from run to run.  Every wait is bounded (~1 s): a rank that
// never signals sets KLG_STATUS_TIMEOUT_PEER and the kernels return without touching dW.
//
// Per-rank buffer (cudaMalloc'd by its rank, opened by the others over CUDA IPC: plain peer
// mappings): [inbox: world x 2 x rows_per_owner x H fp32][final: rows_per_owner x H fp32]
// [flags: 2 x XR_MAX_WORLD uint32, split records: XR_MAX_WORLD x 4 int32; 256 bytes].
#pragma once
#include "klg_kernels.cuh"

namespace klg {

struct XrSync {
  int world, rank, rows_per_owner, hidden, vocab;
  uint32_t epoch;
  float* inbox;                              // this rank's inbox
  float* inbox_peer[XR_MAX_WORLD];           // every rank's inbox (peer pointers; the GEMM's targets)
  float* final_rows;                         // this rank's summed rows [rows_per_owner][H]
  const float* final_peer[XR_MAX_WORLD];     // every rank's summed rows (peer pointers)
  uint32_t* flags;                           // this rank's flags [2][XR_MAX_WORLD]
  uint32_t* flags_peer[XR_MAX_WORLD];        // every rank's flags (peer pointers)
  float* dw;                                 // [V][H] this rank's result
  int stall;                                 // test hook: 1 = wait for a phase nobody signals
  // which of this rank's dW rows have a second K half (slot 1): the chunks before last_start
  // when split_full, the last chunk when split_last.  A split chunk's GEMM writes every row of
  // its slot 1, so slot 1 needs no clearing; each rank publishes this record (its own chunking,
  // from its own row count) to every owner before its first signal, and owners read slot 1 of
  // a source rank only where that rank's record says it was written.
  int cols, last_start, split_full, split_last;
};

// Flag area of a rank's buffer: flags [2][XR_MAX_WORLD] u32, then one split record (4 ints:
// cols, last_start, split_full, split_last) per source rank.
constexpr int XR_REC_OFF = 2 * XR_MAX_WORLD;   // in u32 units from the flags

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Block 0 publishes epoch e in slot [phase][rank] of every rank's flags; every block then waits
// (thread 0, bounded) until every other rank has published e in its own [phase][*] -- no block
// waits on another block of its grid, so the grid may be larger than what is resident.
// Returns the block-uniform outcome.
__device__ __forceinline__ bool xr_signal_wait(const XrSync& x, int phase) {
  __shared__ int ok_s;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (phase == 0)   // this rank's split record, ordered before its signal by the release below
      for (int p = 0; p < x.world; ++p) {
        uint32_t* r = x.flags_peer[p] + XR_REC_OFF + 4 * x.rank;
        r[0] = (uint32_t)x.cols;
        r[1] = (uint32_t)x.last_start;
        r[2] = (uint32_t)x.split_full;
        r[3] = (uint32_t)x.split_last;
      }
    __threadfence_system();
    for (int p = 0; p < x.world; ++p) st_release_sys_u32(x.flags_peer[p] + phase * XR_MAX_WORLD + x.rank, x.epoch);
  }
  if (threadIdx.x == 0) {
    const uint32_t want = x.stall ? x.epoch + 0x40000000u : x.epoch;   // stall: an epoch nobody publishes
    bool ok = true;
    const long long t0 = clock64();
    for (int p = 0; ok && p < x.world; ++p)   // this rank's own work is ordered by the stream
      while ((p != x.rank || x.stall) && (int32_t)(ld_acquire_sys_u32(x.flags + phase * XR_MAX_WORLD + p) - want) < 0) {
        if (clock64() - t0 > KLG_WAIT_CYCLES) {
          atomicOr(&g_status, KLG_STATUS_TIMEOUT_PEER);
          ok = false;
          break;
        }
      }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// Elements (float4) per thread and grid-stride step of the two kernels: independent loads in
// flight per thread, so the loops are bound by bandwidth (HBM for the reduce, NVLink for the
// gather) rather than by one load's latency at a time.
constexpr int XR_U = 8;

__global__ void __launch_bounds__(256) xr_reduce_kernel(const XrSync x) {
  pdl_enter();
  if (!xr_signal_wait(x, 0)) return;
  __shared__ int rec_last[XR_MAX_WORLD], rec_full[XR_MAX_WORLD], rec_lastsplit[XR_MAX_WORLD];
  if (threadIdx.x < x.world) {   // every source rank's split record (published before its signal)
    const uint32_t* r = x.flags + XR_REC_OFF + 4 * threadIdx.x;
    rec_last[threadIdx.x] = (int)ld_acquire_sys_u32(r + 1);
    rec_full[threadIdx.x] = (int)ld_acquire_sys_u32(r + 2);
    rec_lastsplit[threadIdx.x] = (int)ld_acquire_sys_u32(r + 3);
  }
  __syncthreads();
  const int h4 = x.hidden / 4;
  const long long n4 = (long long)x.rows_per_owner * h4;
  const size_t slot_stride = (size_t)x.rows_per_owner * h4;   // float4 per slot
  const float4* in4 = reinterpret_cast<const float4*>(x.inbox);
  float4* out4 = reinterpret_cast<float4*>(x.final_rows);
  const long long step = (long long)gridDim.x * blockDim.x * XR_U;
  for (long long e0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * XR_U; e0 < n4; e0 += step) {
    // the XR_U elements lie in one row (h4 is a multiple of 2; rows are processed whole when
    // h4 % XR_U == 0) or in consecutive rows: each element checks its own row
    float4 acc[XR_U];
    bool live[XR_U];
    int vrow[XR_U];
#pragma unroll
    for (int u = 0; u < XR_U; ++u) {
      acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      const long long e = e0 + u;
      const int orow = (int)(e / h4);
      vrow[u] = ((orow >> 5) * x.world + x.rank) * 32 + (orow & 31);   // global dW row of this own row
      live[u] = e < n4 && vrow[u] < x.vocab;
    }
    for (int src = 0; src < x.world; ++src) {
      bool two[XR_U];   // src wrote a second K half for this row
#pragma unroll
      for (int u = 0; u < XR_U; ++u)
        two[u] = live[u] && (vrow[u] < rec_last[src] ? rec_full[src] : rec_lastsplit[src]) != 0;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const float4* q = in4 + (size_t)(2 * src + half) * slot_stride;
        float4 t[XR_U];
#pragma unroll
        for (int u = 0; u < XR_U; ++u)
          if (half ? two[u] : live[u]) t[u] = q[e0 + u];
#pragma unroll
        for (int u = 0; u < XR_U; ++u)
          if (half ? two[u] : live[u]) {
            acc[u].x += t[u].x;
            acc[u].y += t[u].y;
            acc[u].z += t[u].z;
            acc[u].w += t[u].w;
          }
      }
    }
#pragma unroll
    for (int u = 0; u < XR_U; ++u)
      if (live[u]) out4[e0 + u] = acc[u];
  }
}

// One block: publishes "reduced, epoch e" to every rank and waits (bounded) for every other
// rank's; the copies that follow on the stream then read complete `final` rows.
__global__ void __launch_bounds__(32) xr_wait_kernel(const XrSync x) {
  pdl_enter();
  xr_signal_wait(x, 1);
}

}  // namespace klg
