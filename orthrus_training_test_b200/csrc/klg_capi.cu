// C-ABI of the fused KL-GEMM distillation loss (see include/klgemm.h).
//
// Host side: argument checks, tensor-map construction, work planning and the
// launch sequence.  All device memory is owned by the caller; every entry
// point only enqueues work on the caller's stream and never synchronises
// (except klg_device_status, which reads the device status word).
#include <cuda_runtime.h>
#include <cuda.h>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <algorithm>
#include <functional>
#include <map>
#include <mutex>
#include <queue>
#include <tuple>
#include <vector>

#include <nvtx3/nvToolsExt.h>   // header-only; ranges are free unless a profiler is attached

#include "klg_kernels.cuh"
#include "klg_attn.cuh"
#include "klg_dzt.cuh"
#include "klg_dzi.cuh"
#include "klg_xr.cuh"
#include "klgemm.h"

namespace {

thread_local char g_err[512] = "";
std::atomic<long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(KLG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 tensor map, 128-byte (default) or 64-byte swizzle, zero fill out of bounds.
// inner = contiguous extent (elements), outer = row count, ld = row stride (elements).
// A map is a pure function of these arguments, so encoded maps are kept in a small cache
// (round-robin replacement) keyed by all of them: a decode loop re-encodes nothing for its
// fixed lm_head weight and its reused activation buffers.
struct MapKey {
  const void* base;
  uint64_t inner, outer, ld;
  uint32_t box_inner, box_outer;
  int swz, dt;
  bool operator==(const MapKey& o) const {
    return base == o.base && inner == o.inner && outer == o.outer && ld == o.ld && box_inner == o.box_inner &&
           box_outer == o.box_outer && swz == o.swz && dt == o.dt;
  }
};
struct MapCache {
  static constexpr int kSlots = 64;
  std::mutex mu;
  MapKey key[kSlots];
  CUtensorMap map[kSlots];
  bool used[kSlots] = {};
  int next = 0;
};
MapCache g_maps;

bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
              uint32_t box_outer, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B,
              CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  const MapKey k{base, inner, outer, ld, box_inner, box_outer, (int)swz, (int)dt};
  {
    std::lock_guard<std::mutex> lk(g_maps.mu);
    for (int i = 0; i < MapCache::kSlots; ++i)
      if (g_maps.used[i] && g_maps.key[i] == k) {
        *m = g_maps.map[i];
        return true;
      }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const uint64_t esize = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * esize};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  if (fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  std::lock_guard<std::mutex> lk(g_maps.mu);
  const int i = g_maps.next;
  g_maps.next = (i + 1) % MapCache::kSlots;
  g_maps.key[i] = k;
  g_maps.map[i] = *m;
  g_maps.used[i] = true;
  return true;
}

// 3-D bf16 tensor map {inner, mid, outer} with row strides in elements, 128-byte swizzle,
// zero fill past every extent (not cached: encoded once per call).
bool make_map_3d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t mid, uint64_t outer, uint64_t ld_mid,
                 uint64_t ld_outer, uint32_t box_inner, uint32_t box_mid) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {inner, mid, outer};
  cuuint64_t strides[2] = {ld_mid * 2, ld_outer * 2};
  cuuint32_t box[3] = {box_inner, box_mid, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per-launch timing trace (klg_trace_begin / klg_trace_end).
struct Trace {
  std::mutex mu;
  bool on = false;
  int cap = 0;
  int used = 0;
  std::vector<cudaEvent_t> ev;  // 2 per launch
  std::vector<int> kind;
};
Trace g_trace;

// Records the "before" event of the next traced launch; returns its slot or -1.
int trace_pre(cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_trace.mu);
  if (!g_trace.on || g_trace.used >= g_trace.cap) return -1;
  const int i = g_trace.used++;
  cudaEventRecord(g_trace.ev[2 * i], s);
  return i;
}
void trace_post(int slot, cudaStream_t s, int kind) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lk(g_trace.mu);
  cudaEventRecord(g_trace.ev[2 * slot + 1], s);
  g_trace.kind[slot] = kind;
}

// NVTX range around an entry point or pass, visible in Nsight timelines.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// SMs the persistent kernels leave free (klg_set_sm_reserve): room for communication kernels
// (e.g. an NCCL all-reduce of finished gradient slices) to run beside them.
std::atomic<int> g_sm_reserve{0};

int device_sms() {
  static std::atomic<int> cache[64];   // per device, 0 = not read yet
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && (n = cache[dev].load(std::memory_order_relaxed)) > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// SMs the kernels plan for: the device's, minus the reserve (kept even: CTA pairs).
int num_sms() {
  const int n = device_sms() - g_sm_reserve.load(std::memory_order_relaxed);
  return n < 2 ? 2 : (n & ~1);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Makes the device that owns `p` current on this host thread (binding its
// primary context).  Callers may run on threads that never touched the CUDA
// runtime (e.g. the autograd engine's device thread), where the driver-level
// calls below (tensor-map encoding) would otherwise find no context.  Also
// rejects pointers that are not device memory.
int bind_device(const void* p) {
  cudaPointerAttributes at;
  cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(e, "cudaPointerGetAttributes");
  }
  if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
    return fail(KLG_ERR_ARG, "pointer %p is not device memory", p);
  e = cudaSetDevice(at.device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return KLG_OK;
}

inline int cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }

// Work split of a dual-view launch: n_rt row tiles x n_vt vocab tiles are cut
// into units of vpu vocab tiles.  Picks vpu (>= 4 where possible) so the unit
// count fills the SMs in whole waves as closely as possible, preferring the
// largest vpu among near-ties.
void plan_dual(int n_rt, int n_vt, int n_sm, int& vpu, int& n_uv, int max_uv = 64, int min_vpu = 4) {
  const int vmin = n_vt < min_vpu ? n_vt : min_vpu;
  double best = -1.0;
  vpu = n_vt;
  for (int v = n_vt; v >= vmin; --v) {
    const int uv = cdiv(n_vt, v);
    if (uv > max_uv) break;
    const long long units = (long long)n_rt * uv;
    const long long waves = (units + n_sm - 1) / n_sm;
    // balance of tile work across SMs (tiles per unit vary only in the last uv)
    const double eff = (double)n_rt * n_vt / ((double)waves * n_sm * v);
    if (eff > best + 0.005) {
      best = eff;
      vpu = v;
    }
  }
  n_uv = cdiv(n_vt, vpu);
}

int gemm_bn(long long hidden) {
  if (hidden % 256 == 0) return 256;
  if (hidden % 192 == 0) return 192;
  if (hidden % 128 == 0) return 128;
  return 256;
}

template <typename Kern>
cudaError_t set_smem(Kern k, int bytes) {
  // once per (kernel, device, size): the attribute persists in the context
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_tuple(reinterpret_cast<const void*>(k), dev, bytes);
  std::lock_guard<std::mutex> lk(mu);
  if (std::find(done.begin(), done.end(), key) != done.end()) return cudaSuccess;
  e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.push_back(key);
  return e;
}

// Programmatic dependent launch (on unless KLG_PDL=0): each launch may start its set-up
// while the previous kernel in the stream drains; the kernels wait (griddepcontrol.wait)
// before touching global memory.
bool pdl_on() {
  static const bool on = [] {
    const char* v = std::getenv("KLG_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Launch with an optional cluster of `cluster` CTAs and programmatic stream serialisation.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t s, int cluster,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_on()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

template <int EPI>
int launch_lse_pair(const CUtensorMap& mhs, const CUtensorMap& mht, const CUtensorMap& mw, const klg::LseArgs& a,
                    cudaStream_t s) {
  // A resident across the unit's tiles when it fits -- except for replicated rows (a handful
  // of rows, W streamed once from HBM), where the streamed-A ring's six W stages in flight
  // measured 2-4 us faster than the resident ring's four (32-128 rows, H=576, V=49153)
  const bool res = a.n_kb <= klg::LSE_RES_MAX_KB && a.rep == 1;
  auto k = res ? klg::lse_pair_kernel<true, EPI> : klg::lse_pair_kernel<false, EPI>;
  const int smem = res ? klg::LSE_RES_SMEM : klg::LSE_SMEM;
  cudaError_t e = set_smem(k, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(lse_pair_kernel)");
  const int pairs = a.n_units < num_sms() / 2 ? a.n_units : num_sms() / 2;
  const int slot = trace_pre(s);
  e = launch_k(k, dim3(2 * pairs), dim3(klg::LSE_THREADS), smem, s, 2, mhs, mht, mw, a);
  trace_post(slot, s, EPI == klg::EPI_LSE ? KLG_KIND_STATS : KLG_KIND_SAMPLE);
  if (e != cudaSuccess) return cuda_fail(e, "launch lse_pair_kernel");
  ++g_launches;
  return KLG_OK;
}

// The resident-student-row variant (H <= 576) measured slower than the streamed kernel at the
// 16,384-row shape (dZ chunk 0.66 vs 0.51 ms: its five 12 KB stages hide ~1,300 cycles of load
// latency against the streamed ring's ~2,600), so it runs only with KLG_DZ_RES=1.
bool dual_res_on(int n_kb) {
  static const bool on = [] {
    const char* v = std::getenv("KLG_DZ_RES");
    return v && v[0] == '1';
  }();
  return on && n_kb <= klg::DZR_MAX_KB;
}

// Tensor maps of a dual-view launch: h_s with 128 x 64 boxes; h_t and W with 128 x 64 / 64 x 64
// boxes (128-byte swizzle), or 128 x 32 / 64 x 32 (64-byte swizzle) for the resident variant.
bool dual_maps(const void* hs, const void* ht, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab, bool res,
               CUtensorMap* mhs, CUtensorMap* mht, CUtensorMap* mw) {
  if (!make_map(mhs, hs, hidden, n_rows, hidden, klg::BK, klg::BM)) return false;
  if (res)
    return make_map(mht, ht, hidden, n_rows, hidden, klg::DZR_SUB, klg::BM, CU_TENSOR_MAP_SWIZZLE_64B) &&
           make_map(mw, w, hidden, vocab, hidden, klg::DZR_SUB, klg::DZP_BN / 2, CU_TENSOR_MAP_SWIZZLE_64B);
  return make_map(mht, ht, hidden, n_rows, hidden, klg::BK, klg::BM) &&
         make_map(mw, w, hidden, vocab, hidden, klg::BK, klg::DZP_BN / 2);
}

template <int MODE>
int launch_dual_pair(const CUtensorMap& mhs, const CUtensorMap& mht, const CUtensorMap& mw, const CUtensorMap& mout,
                     const CUtensorMap& mout2, const klg::DualArgs& a, cudaStream_t s, bool split = false) {
  const bool res = !split && dual_res_on(a.n_kb);
  auto k = split ? klg::dual_pair_kernel<MODE, false, true>
                 : (res ? klg::dual_pair_kernel<MODE, true> : klg::dual_pair_kernel<MODE, false>);
  const int smem = res ? klg::DualResCfg<MODE>::SMEM : klg::DZP_SMEM;
  const int threads = res ? klg::DZR_THREADS : klg::DZP_THREADS;
  cudaError_t e = set_smem(k, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(dual_pair_kernel)");
  const int pairs = a.n_units < num_sms() / 2 ? a.n_units : num_sms() / 2;
  const int slot = trace_pre(s);
  e = launch_k(k, dim3(2 * pairs), dim3(threads), smem, s, 2, mhs, mht, mw, mout, mout2, a);
  trace_post(slot, s, MODE == klg::MODE_DZ ? KLG_KIND_DZ : KLG_KIND_STATS);
  if (e != cudaSuccess) return cuda_fail(e, "launch dual_pair_kernel");
  ++g_launches;
  return KLG_OK;
}

// The transposed dZ kernel (klg_dzt.cuh) runs only with KLG_DZT=1 (A/B timing).  Its main loop
// moves 20 % fewer (streamed W) to 60 % fewer (resident W) bytes per MMA cycle than the
// row-major kernel, but its epilogue -- per-column row constants and a cross-lane reduction of
// the KL cross term -- takes ~10k cycles a tile.  Measured dZ time per training step, transposed
// / row-major / interleaved-view kernel: H = 2048: 20.5 / 21.3 / 19.0 ms; H = 1024: 30.8 / 26.1
// / 24.0 ms; H = 576: 1.82 / 1.44 / 1.41 ms.  The interleaved-view kernel is the default.
bool dzt_on(int64_t hidden) {
  static const bool force = [] {
    const char* v = std::getenv("KLG_DZT");
    return v && v[0] == '1';
  }();
  (void)hidden;
  return force;
}

inline int64_t round8(int64_t x) { return (x + 7) & ~int64_t(7); }

// The interleaved-view dZ kernel (klg_dzi.cuh) replaces the row-major one on the bf16 path
// wherever the transposed kernel is not used.  KLG_DZI=0 keeps the row-major kernel (A/B
// timing); KLG_DZI=2 makes a rejected interleaved map an error instead of a fallback (tests);
// KLG_DZI=3 uses the row-interleaved layout even where the 8-row-group one applies (tests).
int dzi_mode() {
  static const int mode = [] {
    const char* v = std::getenv("KLG_DZI");
    return v ? (v[0] == '0' ? 0 : v[0] == '2' ? 2 : v[0] == '3' ? 3 : 1) : 1;
  }();
  return mode;
}
bool dzi_on() { return dzi_mode() > 0; }

// Tensor map of both views interleaved along M, over the lower of the two base pointers with
// the distance between the bases as the view stride; *s_view = the student's view index.
//  *lay = DZI_G8_S0 / _S1 (N % 8 == 0): dims {H, 8 rows, 2 views, N / 8 groups}, strides {2H
//    bytes, gap, 16H bytes}; a {64, 8, 2, 8} box lands as 128 rows in (group, view, row) order.
//  *lay = DZI_ROW: dims {H, 2 views, N rows}, strides {gap, 2H bytes}; a {64, 2, 64} box lands
//    as 128 rows in (token row, view) order.
// Fails (the caller keeps the row-major kernel) when both views are the same tensor or the
// driver rejects the strides.
bool dzi_map(CUtensorMap* m, const void* hs, const void* ht, int64_t n_rows, int64_t hidden, int* s_view, int* lay) {
  const uintptr_t ps = reinterpret_cast<uintptr_t>(hs), pt = reinterpret_cast<uintptr_t>(ht);
  if (ps == pt) return false;
  const uint64_t gap = ps < pt ? pt - ps : ps - pt;
  if (gap % 16 != 0 || gap >= (1ull << 40)) return false;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  *s_view = ps < pt ? 0 : 1;
  void* base = const_cast<void*>(ps < pt ? hs : ht);
  const cuuint64_t rowb = (cuuint64_t)hidden * 2;
  if (n_rows % 8 == 0 && dzi_mode() != 3) {
    *lay = *s_view == 0 ? klg::DZI_G8_S0 : klg::DZI_G8_S1;
    cuuint64_t dims[4] = {(cuuint64_t)hidden, 8, 2, (cuuint64_t)(n_rows / 8)};
    cuuint64_t strides[3] = {rowb, gap, 8 * rowb};
    cuuint32_t box[4] = {klg::BK, 8, 2, klg::DZI_ROWS / 16};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  *lay = klg::DZI_ROW;
  cuuint64_t dims[3] = {(cuuint64_t)hidden, 2, (cuuint64_t)n_rows};
  cuuint64_t strides[2] = {gap, rowb};
  cuuint32_t box[3] = {klg::BK, 2, klg::DZI_ROWS / 2};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_dzi(int lay, const CUtensorMap& mh, const CUtensorMap& mw, const CUtensorMap& mout, const klg::DziArgs& a,
               cudaStream_t s) {
  auto k = lay == klg::DZI_G8_S0 ? klg::dzi_pair_kernel<klg::DZI_G8_S0>
                                 : lay == klg::DZI_G8_S1 ? klg::dzi_pair_kernel<klg::DZI_G8_S1>
                                                         : klg::dzi_pair_kernel<klg::DZI_ROW>;
  cudaError_t e = set_smem(k, klg::DZI_SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(dzi_pair_kernel)");
  const int pairs = a.n_units < num_sms() / 2 ? a.n_units : num_sms() / 2;
  const int slot = trace_pre(s);
  e = launch_k(k, dim3(2 * pairs), dim3(klg::DZI_THREADS), klg::DZI_SMEM, s, 2, mh, mw, mout, a);
  trace_post(slot, s, KLG_KIND_DZ);
  if (e != cudaSuccess) return cuda_fail(e, "launch dzi_pair_kernel");
  ++g_launches;
  return KLG_OK;
}

// Work split of a transposed dZ launch: units of g vocab pair tiles x rpu row tiles.  Picks
// the split that fills the pairs in whole waves best, then the most row tiles per unit (the
// reuse of a resident W tile), then the most vocab tiles per unit (fewer cross-term partial
// rows), with the partial rows of the whole pass (n_chunks launches) kept within 64 MiB.
struct DztPlan {
  int g, rpu, n_vg, n_rg;
};
DztPlan plan_dzt(int n_vp, int n_rt, int pairs, int64_t n_rows, int n_chunks) {
  DztPlan best{1, 1, n_vp, n_rt};
  double best_eff = -1.0;
  const int64_t cap_rows = std::max<int64_t>(2, (64ll << 20) / (4 * n_rows * std::max(1, n_chunks)));
  for (int rpu = klg::DZT_RPU_MAX; rpu >= 1; rpu >>= 1) {
    for (int g = 1; g <= 64; g <<= 1) {
      const int n_vg = cdiv(n_vp, g), n_rg = cdiv(n_rt, rpu);
      const bool last_g = g >= n_vp;
      if (2ll * n_vg > cap_rows && !last_g) continue;
      const long long units = (long long)n_vg * n_rg;
      const long long waves = (units + pairs - 1) / pairs;
      const double eff = (double)n_vp * n_rt / ((double)waves * pairs * g * rpu);
      if (eff > best_eff + 0.02) {
        best_eff = eff;
        best = DztPlan{g, rpu, n_vg, n_rg};
      }
      if (last_g) break;
    }
  }
  return best;
}

int launch_dzt(const CUtensorMap& mw, const CUtensorMap& mhs, const CUtensorMap& mht, const CUtensorMap& mout,
               const klg::DztArgs& a, cudaStream_t s) {
  const bool res = a.n_kb <= klg::DZT_MAX_KB;
  auto k = res ? klg::dzt_pair_kernel<true> : klg::dzt_pair_kernel<false>;
  const int smem = res ? klg::DztCfg<true>::SMEM : klg::DztCfg<false>::SMEM;
  cudaError_t e = set_smem(k, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(dzt_pair_kernel)");
  const int pairs = a.n_units < num_sms() / 2 ? a.n_units : num_sms() / 2;
  const int slot = trace_pre(s);
  e = launch_k(k, dim3(2 * pairs), dim3(klg::DZT_THREADS), smem, s, 2, mw, mhs, mht, mout, a);
  trace_post(slot, s, KLG_KIND_DZ);
  if (e != cudaSuccess) return cuda_fail(e, "launch dzt_pair_kernel");
  ++g_launches;
  return KLG_OK;
}

// Longest-first greedy assignment of tiles [t_begin, t_end) to `pairs` CTA pairs.
// Cost of a tile in k-block units: its K range plus the epilogue and pipeline refill.
constexpr int kTileOverheadKb = 4;

int tile_kb(const klg::GemmProblem& P, int local) {
  if (P.n_split == 1) return P.n_kb;
  return local < P.n_mt * P.n_nt ? P.kb_split : P.n_kb - P.kb_split;
}

// Longest-processing-time-first assignment of tiles [t_begin, t_end) to `pairs` CTA pairs.
// Returns the makespan in k-block units; fills `lists` when given.
long long lpt_assign(const klg::PairGemmArgs& g, int t_begin, int t_end, int pairs,
                     std::vector<std::vector<uint32_t>>* lists) {
  std::vector<std::pair<int, uint32_t>> order;   // (cost, tile)
  order.reserve(t_end - t_begin);
  for (int t = t_begin; t < t_end; ++t) {
    const int pi = t < g.p[0].n_tiles ? 0 : 1;
    order.push_back({tile_kb(g.p[pi], pi ? t - g.p[0].n_tiles : t) + kTileOverheadKb, (uint32_t)t});
  }
  std::stable_sort(order.begin(), order.end(), [](const std::pair<int, uint32_t>& x, const std::pair<int, uint32_t>& y) {
    return x.first > y.first;
  });
  typedef std::pair<long long, int> Load;   // (assigned cost, pair)
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < pairs; ++c) heap.push(Load(0, c));
  long long makespan = 0;
  for (const auto& o : order) {
    Load l = heap.top();
    heap.pop();
    if (lists) (*lists)[l.second].push_back(o.second);
    l.first += o.first;
    makespan = std::max(makespan, l.first);
    heap.push(l);
  }
  return makespan;
}

void build_schedule(const klg::PairGemmArgs& g, int t_begin, int t_end, int pairs, klg::PairSchedule& sc) {
  std::vector<std::vector<uint32_t>> lists(pairs);
  lpt_assign(g, t_begin, t_end, pairs, &lists);
  int n = 0;
  for (int c = 0; c < pairs; ++c) {
    sc.start[c] = (uint16_t)n;
    for (uint32_t t : lists[c]) sc.tile[n++] = t;
  }
  sc.start[pairs] = (uint16_t)n;
}

template <int BN>
int launch_gemm_pair_t(const CUtensorMap& a0, const CUtensorMap& b0, const CUtensorMap& a1, const CUtensorMap& b1,
                       const CUtensorMap& c0, const CUtensorMap& c1, const klg::PairGemmArgs& g, cudaStream_t s,
                       const klg::XrMaps& xm) {
  using Cfg = klg::PairGemmCfg<BN>;
  auto k = klg::gemm_pair_kernel<BN>;
  cudaError_t e = set_smem(k, Cfg::SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm_pair_kernel)");
  const int max_pairs = std::min(num_sms() / 2, klg::PAIR_MAX_CLUSTERS);
  static thread_local klg::PairSchedule sc;   // 25 KB: kept off the stack
  for (int t0 = 0; t0 < g.n_tiles; t0 += klg::PAIR_MAX_TILES) {
    const int t1 = std::min(g.n_tiles, t0 + klg::PAIR_MAX_TILES);
    const int pairs = std::min(max_pairs, t1 - t0);
    build_schedule(g, t0, t1, pairs, sc);
    const int slot = trace_pre(s);
    e = launch_k(k, dim3(2 * pairs), dim3(Cfg::THREADS), Cfg::SMEM, s, 2, a0, b0, a1, b1, c0, c1, g, sc, xm);
    trace_post(slot, s, KLG_KIND_GEMM);
    if (e != cudaSuccess) return cuda_fail(e, "launch gemm_pair_kernel");
    ++g_launches;
  }
  return KLG_OK;
}

int launch_gemm_pair(int bn, const CUtensorMap& a0, const CUtensorMap& b0, const CUtensorMap& a1, const CUtensorMap& b1,
                     const CUtensorMap& c0, const CUtensorMap& c1, const klg::PairGemmArgs& g, cudaStream_t s,
                     const klg::XrMaps* xm = nullptr) {
  static const klg::XrMaps none{};   // unused unless g.xr is set
  const klg::XrMaps& m = xm ? *xm : none;
  switch (bn) {
    case 128: return launch_gemm_pair_t<128>(a0, b0, a1, b1, c0, c1, g, s, m);
    case 192: return launch_gemm_pair_t<192>(a0, b0, a1, b1, c0, c1, g, s, m);
    default: return launch_gemm_pair_t<256>(a0, b0, a1, b1, c0, c1, g, s, m);
  }
}

// kb_split: 0 = no K split; else the first of two K pieces has kb_split k-blocks.
klg::GemmProblem gemm_problem(bool on, int M, int Ncol, int K, int bn, float* C, int ldc, int accumulate, int a_k0,
                              int b_k0, int a_mn, int bm = klg::BM, int kb_split = 0, int c_row0 = 0) {
  klg::GemmProblem g{};
  g.M = M;
  g.Ncol = Ncol;
  g.K = K;
  g.n_mt = cdiv(M, bm);
  g.n_nt = cdiv(Ncol, bn);
  g.n_kb = cdiv(K, klg::BK);
  g.n_split = (kb_split > 0 && kb_split < g.n_kb) ? 2 : 1;
  g.kb_split = g.n_split == 2 ? kb_split : g.n_kb;
  g.c_row0 = c_row0;
  g.n_tiles = on ? g.n_mt * g.n_nt * g.n_split : 0;
  g.C = C;
  g.ldc = ldc;
  g.accumulate = accumulate;
  g.a_k0 = a_k0;
  g.b_k0 = b_k0;
  g.a_mn = a_mn;
  return g;
}

// Split point of dW's K for one backward chunk (0 = no split): the candidate whose
// longest-first schedule has the shortest makespan, memoised per shape.
int pick_dw_split(int n_rows, int wv, int hidden, int bn) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int>, int> memo;
  const int pairs = std::min(num_sms() / 2, klg::PAIR_MAX_CLUSTERS);
  const auto key = std::make_tuple(n_rows, wv, hidden, bn, pairs);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
  }
  klg::PairGemmArgs g{};
  g.p[1] = gemm_problem(true, n_rows, hidden, wv, bn, nullptr, hidden, 1, 0, 0, 0, 256, 0, 0);
  const int dw_kb = cdiv(n_rows, klg::BK);
  std::vector<int> cands(1, 0);
  for (int c = (dw_kb + 1) / 2; c < dw_kb; c += 4) cands.push_back(c);
  long long best = -1;
  int pick = 0;
  for (int c : cands) {
    g.p[0] = gemm_problem(true, wv, hidden, n_rows, bn, nullptr, hidden, 1, 0, 0, 1, 256, c, 0);
    g.n_tiles = g.p[0].n_tiles + g.p[1].n_tiles;
    if (g.n_tiles > klg::PAIR_MAX_TILES) continue;
    const long long m = lpt_assign(g, 0, g.n_tiles, std::min(pairs, g.n_tiles), nullptr);
    if (best < 0 || m < best) {
      best = m;
      pick = c;
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  memo[key] = pick;
  return pick;
}

int check_problem(const void* hs, const void* ht, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab,
                  float inv_temp) {
  if (!hs || !ht || !w) return fail(KLG_ERR_ARG, "null input pointer");
  if (n_rows < 1 || hidden < 8 || vocab < 1) return fail(KLG_ERR_ARG, "bad shape N=%lld H=%lld V=%lld",
                                                          (long long)n_rows, (long long)hidden, (long long)vocab);
  if (n_rows > (1ll << 30) || hidden > (1ll << 20) || vocab > (1ll << 30))
    return fail(KLG_ERR_ARG, "shape too large N=%lld H=%lld V=%lld", (long long)n_rows, (long long)hidden,
                (long long)vocab);
  if (hidden % 8 != 0) return fail(KLG_ERR_ALIGN, "hidden=%lld must be a multiple of 8", (long long)hidden);
  // the tensor-core kernels load 64-column k-blocks; hidden sizes below one k-block (narrower
  // rows than the TMA box) are outside what they are built and tested for
  if (hidden < 64) return fail(KLG_ERR_ARG, "hidden=%lld: the lm_head kernels need hidden >= 64", (long long)hidden);
  if (!aligned16(hs) || !aligned16(ht) || !aligned16(w)) return fail(KLG_ERR_ALIGN, "inputs must be 16-byte aligned");
  if (!(inv_temp > 0.f) || !std::isfinite(inv_temp)) return fail(KLG_ERR_ARG, "inv_temp must be finite and > 0");
  return KLG_OK;
}

}  // namespace

// ======================================================================= C-ABI
extern "C" {

int klg_version(void) { return KLG_VERSION; }

int klg_last_error(char* buf, int len) {
  if (!buf || len <= 0) return KLG_ERR_ARG;
  std::snprintf(buf, (size_t)len, "%s", g_err);
  return KLG_OK;
}

int klg_device_status(int* status, int reset) {
  if (!status) return fail(KLG_ERR_ARG, "null status pointer");
  cudaError_t e = cudaMemcpyFromSymbol(status, klg::g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "read device status");
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(klg::g_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "reset device status");
  }
  return KLG_OK;
}

long long klg_launch_count(void) { return g_launches.load(); }

int klg_set_sm_reserve(int n_sms) {
  if (n_sms < 0 || n_sms > 64) return fail(KLG_ERR_ARG, "SM reserve %d out of range [0, 64]", n_sms);
  g_sm_reserve.store(n_sms, std::memory_order_relaxed);
  return KLG_OK;
}

int klg_selftest_wait_timeout(void* stream) {
  cudaError_t e = launch_k(klg::wait_selftest_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, 1);
  if (e != cudaSuccess) return cuda_fail(e, "launch wait_selftest_kernel");
  ++g_launches;
  return KLG_OK;
}

// Forward statistics run on CTA pairs: (256-row pair tile, vocab range) units, at most 8
// vocab ranges per row, one partial record per unit and epilogue column slice.
constexpr int kStatsMaxRanges = 8;

// Vocab ranges of the forward statistics: planned on the interleaved kernel's units (128-row
// pair tiles x 256-column vocab tiles; vpu vocab tiles per range) unless KLG_DZI=0 keeps the
// row-major kernel's (256-row tiles x 128 columns).  Where the row-major kernel runs under the
// interleaved plan it takes 2 * vpu of its 128-column tiles per range: the same number of ranges.
void stats_plan(int64_t n_rows, int64_t vocab, int& vpu, int& n_uv) {
  if (dzi_on())
    plan_dual(cdiv(n_rows, klg::DZI_ROWS), cdiv(vocab, klg::DZI_BN), num_sms() / 2, vpu, n_uv, kStatsMaxRanges);
  else
    plan_dual(cdiv(n_rows, 256), cdiv(vocab, klg::DZP_BN), num_sms() / 2, vpu, n_uv, kStatsMaxRanges);
}

int klg_num_partials(int64_t n_rows, int64_t vocab, int* n_part) {
  if (!n_part || n_rows < 1 || vocab < 1) return fail(KLG_ERR_ARG, "bad arguments to klg_num_partials");
  int vpu, n_uv;
  stats_plan(n_rows, vocab, vpu, n_uv);
  *n_part = n_uv * klg::DZP_CSPLIT;
  return KLG_OK;
}

int klg_fwd_stats(const void* hs, const void* ht, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab,
                  float inv_temp, float* partials, int n_part, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!partials || !aligned16(partials)) return fail(KLG_ERR_ARG, "partials must be non-null and 16-byte aligned");
  if (n_part < klg::DZP_CSPLIT || n_part % klg::DZP_CSPLIT != 0 || n_part > kStatsMaxRanges * klg::DZP_CSPLIT)
    return fail(KLG_ERR_ARG, "n_part=%d is not a record count this kernel writes (use klg_num_partials)", n_part);
  if ((rc = bind_device(hs))) return rc;   // the exact plan below depends on the SM count of hs's device
  int vpu, n_uv;
  stats_plan(n_rows, vocab, vpu, n_uv);
  if (n_part != n_uv * klg::DZP_CSPLIT)
    return fail(KLG_ERR_ARG, "n_part=%d but this device plans %d (use klg_num_partials)", n_part, n_uv * klg::DZP_CSPLIT);
  NvtxRange nvtx_range("klg_fwd_stats");
  // interleaved-view statistics (8-row groups: N % 8 == 0, two distinct tensors)
  if (dzi_on() && n_rows % 8 == 0 && hs != ht) {
    alignas(64) CUtensorMap mhi, mw256;
    int s_view = 0, lay = klg::DZI_ROW;
    if (dzi_map(&mhi, hs, ht, n_rows, hidden, &s_view, &lay) && lay != klg::DZI_ROW &&
        make_map(&mw256, w, hidden, vocab, hidden, klg::BK, klg::DZI_BN / 2)) {
      klg::DziArgs b{};
      b.n_rows = (int)n_rows;
      b.v_begin = 0;
      b.v_count = (int)vocab;
      b.n_rt = cdiv(n_rows, klg::DZI_ROWS);
      b.n_vt = cdiv(vocab, klg::DZI_BN);
      b.vt_per_unit = vpu;
      b.n_units = b.n_rt * n_uv;
      b.n_kb = cdiv(hidden, klg::BK);
      b.s_view = s_view;
      b.scale_log2 = inv_temp * 1.4426950408889634f;
      b.inv_temp = inv_temp;
      b.partials = partials;
      auto k = lay == klg::DZI_G8_S0 ? klg::dzi_pair_kernel<klg::DZI_G8_S0, klg::MODE_STATS>
                                     : klg::dzi_pair_kernel<klg::DZI_G8_S1, klg::MODE_STATS>;
      cudaError_t e = set_smem(k, klg::DZI_SMEM);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(dzi_pair_kernel)");
      const int pairs = b.n_units < num_sms() / 2 ? b.n_units : num_sms() / 2;
      const int slot = trace_pre((cudaStream_t)stream);
      e = launch_k(k, dim3(2 * pairs), dim3(klg::DZI_THREADS), klg::DZI_SMEM, (cudaStream_t)stream, 2, mhi, mw256, mw256,
                   b);
      trace_post(slot, (cudaStream_t)stream, KLG_KIND_STATS);
      if (e != cudaSuccess) return cuda_fail(e, "launch dzi_pair_kernel (statistics)");
      ++g_launches;
      return KLG_OK;
    }
    if (dzi_mode() == 2 && lay != klg::DZI_ROW) return fail(KLG_ERR_CUDA, "interleaved-view tensor map rejected (KLG_DZI=2)");
  }
  klg::DualArgs a{};
  a.n_rows = (int)n_rows;
  a.v_begin = 0;
  a.v_count = (int)vocab;
  a.n_rt = cdiv(n_rows, 256);
  a.n_vt = cdiv(vocab, klg::DZP_BN);
  a.vt_per_unit = dzi_on() ? 2 * vpu : vpu;   // same vocab ranges as the plan
  if (cdiv(a.n_vt, a.vt_per_unit) != n_uv) return fail(KLG_ERR_ARG, "internal plan mismatch (statistics ranges)");
  a.n_units = a.n_rt * n_uv;
  a.n_kb = cdiv(hidden, klg::BK);
  a.scale_log2 = inv_temp * 1.4426950408889634f;
  a.partials = partials;
  alignas(64) CUtensorMap mhs, mht, mw;
  if (!dual_maps(hs, ht, w, n_rows, hidden, vocab, dual_res_on(a.n_kb), &mhs, &mht, &mw))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  return launch_dual_pair<klg::MODE_STATS>(mhs, mht, mw, mw, mw, a, (cudaStream_t)stream);
}

int klg_merge_stats(const float* partials, int n_part, int64_t n_rows, float* stats, void* stream) {
  if (!partials || !stats || n_part < 1 || n_rows < 1) return fail(KLG_ERR_ARG, "bad arguments to klg_merge_stats");
  if (int rc = bind_device(partials)) return rc;
  const int slot = trace_pre((cudaStream_t)stream);
  cudaError_t e = launch_k(klg::merge_kernel, dim3(cdiv(n_rows, 256)), dim3(256), 0, (cudaStream_t)stream, 1, partials, n_part,
                           (int)n_rows, stats);
  trace_post(slot, (cudaStream_t)stream, KLG_KIND_MERGE);
  if (e != cudaSuccess) return cuda_fail(e, "launch merge_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_count_valid(const uint8_t* mask, int64_t n_rows, float* count, void* stream) {
  if (!mask || !count || n_rows < 1 || n_rows > (1ll << 30)) return fail(KLG_ERR_ARG, "bad arguments to klg_count_valid");
  if (int rc = bind_device(mask)) return rc;
  const int slot = trace_pre((cudaStream_t)stream);
  cudaError_t e = launch_k(klg::count_valid_kernel, dim3(1), dim3(1024), 0, (cudaStream_t)stream, 1, mask, (int)n_rows, count);
  trace_post(slot, (cudaStream_t)stream, KLG_KIND_COUNT);
  if (e != cudaSuccess) return cuda_fail(e, "launch count_valid_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_finalize(const float* stats, const uint8_t* mask, int64_t n_rows, const float* count, float* loss, float* lse,
                 float* row_kl, void* stream) {
  if (!stats || !mask || !count || !loss || n_rows < 1 || n_rows > (1ll << 30))
    return fail(KLG_ERR_ARG, "bad arguments to klg_finalize");
  if (int rc = bind_device(stats)) return rc;
  const int slot = trace_pre((cudaStream_t)stream);
  cudaError_t e = launch_k(klg::finalize_kernel, dim3(1), dim3(1024), 0, (cudaStream_t)stream, 1, stats, mask, (int)n_rows, count, loss,
                           lse, row_kl);
  trace_post(slot, (cudaStream_t)stream, KLG_KIND_FINALIZE);
  if (e != cudaSuccess) return cuda_fail(e, "launch finalize_kernel");
  ++g_launches;
  return KLG_OK;
}

int64_t klg_fwd_workspace_bytes(int64_t n_rows, int64_t vocab) {
  int n_part = 0;
  if (klg_num_partials(n_rows, vocab, &n_part) != KLG_OK) return -1;
  return (int64_t)(n_part + 1) * 5 * n_rows * 4 + 256;
}

int klg_fwd(const void* hs, const void* ht, const void* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
            int64_t vocab, float inv_temp, int count_given, float* count, float* loss, float* lse, float* row_kl,
            void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !count || !loss || !lse) return fail(KLG_ERR_ARG, "null output pointer");
  // at least one vocab range (DZP_CSPLIT records) plus the merged record: checked before any device call
  if (!workspace || workspace_bytes < (int64_t)(klg::DZP_CSPLIT + 1) * 5 * n_rows * 4 || !aligned16(workspace))
    return fail(KLG_ERR_WORKSPACE, "forward workspace needs at least %lld bytes (16-byte aligned)",
                (long long)(klg::DZP_CSPLIT + 1) * 5 * n_rows * 4);
  if ((rc = bind_device(hs))) return rc;   // the partial-record count depends on hs's device
  int n_part = 0;
  if ((rc = klg_num_partials(n_rows, vocab, &n_part))) return rc;
  const int64_t need = (int64_t)(n_part + 1) * 5 * n_rows * 4;
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(KLG_ERR_WORKSPACE, "forward workspace needs %lld bytes (16-byte aligned)", (long long)need);
  NvtxRange nvtx_range("klg_fwd");
  float* parts = static_cast<float*>(workspace);
  float* stats = parts + (size_t)n_part * 5 * n_rows;
  if (!count_given && (rc = klg_count_valid(mask, n_rows, count, stream))) return rc;
  if ((rc = klg_fwd_stats(hs, ht, w, n_rows, hidden, vocab, inv_temp, parts, n_part, stream))) return rc;
  if ((rc = klg_merge_stats(parts, n_part, n_rows, stats, stream))) return rc;
  return klg_finalize(stats, mask, n_rows, count, loss, lse, row_kl, stream);
}

// Backward workspace: [KLG_BWD_HEADER bytes, reserved][dZ chunk N x C bf16].  The header also
// bounds the chunk count (cdiv(V, C) <= KLG_BWD_HEADER / 4) and, in the fused layout, is
// where the pass-1 partials start; the training step keeps its loss kernel's completion
// counter in the header's first word.
#define KLG_BWD_HEADER 4096

int64_t klg_bwd_chunk_cols(int64_t n_rows, int64_t vocab, int64_t workspace_bytes) {
  if (n_rows < 1 || vocab < 1) return -1;
  const int64_t full = (int64_t)cdiv(vocab, 128) * 128;
  int64_t c = (workspace_bytes - KLG_BWD_HEADER) / (round8(n_rows) * 2);
  c = (c / 128) * 128;
  if (c > full) c = full;
  if (c < 128 || cdiv(vocab, c) > KLG_BWD_HEADER / 4) return -1;
  return c;
}

int64_t klg_bwd_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab) {
  (void)hidden;
  if (n_rows < 1 || vocab < 1) return -1;
  // dZ chunk of up to 512 MiB (at least 2048 columns): fewer, fuller launches beat an
  // L2-resident chunk (measured at the 16k-row shape, pass 2 per step: 64 MiB chunks
  // 3.9 ms, 256 MiB 3.0 ms, 512 MiB 2.9 ms; wider chunks gained nothing more)
  const int64_t full = (int64_t)cdiv(vocab, 128) * 128;
  int64_t cols = (512ll << 20) / (round8(n_rows) * 2);
  cols = (cols / 128) * 128;
  if (cols < 2048) cols = 2048;
  if (cols > full) cols = full;
  while (cdiv(vocab, cols) > KLG_BWD_HEADER / 4) cols += 128;
  return KLG_BWD_HEADER + round8(n_rows) * cols * 2;
}

}  // extern "C"

namespace {

// Pass 2 over vocab chunks of `cols` columns: dZ chunk (dual_pair_kernel<MODE_DZ>) then one
// pair-GEMM launch for dW_chunk and dH.  With a_parts set, the dZ pass also writes the
// per-unit KL cross-term partials (at most 8 units per chunk), returning their count.
// split (the fp32-faithful path): dZ is kept as two bf16 planes (hi and lo, row stride 2 * cols)
// and each chunk's GEMM runs once per plane, both adding into the same fp32 dW and dH; dW's
// K is then never split, so every dW element gets one addend per plane, in plane order.
// chunk_events (optional, n_events of them): event c is recorded on the stream once chunk c's
// GEMM is enqueued, i.e. when dW rows [c * cols, (c + 1) * cols) are final.
int run_pass2(const void* hs, const void* ht, const void* w, const uint8_t* mask, const float* lse, const float* count,
              const float* grad, int64_t n_rows, int64_t hidden, int64_t vocab, float inv_temp, float* d_hs, float* d_w,
              __nv_bfloat16* dz, int64_t cols, float* a_parts, int* n_ap_out, cudaStream_t s, bool split = false,
              void* const* chunk_events = nullptr, int n_events = 0, const klg::XrArgs* xr = nullptr) {
  int rc;
  const bool tr = !split && dzt_on(hidden);           // dZ^T [cols][ld_n] from the transposed kernel
  const int64_t ld_n = round8(n_rows);
  const int64_t ld_dz = split ? 2 * cols : cols;      // row-major dZ [n_rows][ld_dz]
  const int bn = gemm_bn(hidden);
  alignas(64) CUtensorMap mhs, mht, mw, mw_mn, mhs_mn;
  if (tr) {   // W as the A operand (128-row boxes), each CTA's 64-row halves of both views
    if (!make_map(&mw, w, hidden, vocab, hidden, klg::BK, klg::BM) ||
        !make_map(&mhs, hs, hidden, n_rows, hidden, klg::BK, klg::DZT_BN / 2) ||
        !make_map(&mht, ht, hidden, n_rows, hidden, klg::BK, klg::DZT_BN / 2))
      return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  } else if (!dual_maps(hs, ht, w, n_rows, hidden, vocab, dual_res_on(cdiv(hidden, klg::BK)), &mhs, &mht, &mw)) {
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  }
  // interleaved-view dZ kernel: both views through one 3-D map, W in 128-row halves
  alignas(64) CUtensorMap mhi, mw256;
  int s_view = 0, lay = klg::DZI_ROW;
  bool il = false;
  if (!split && !tr && dzi_on() && hs != ht) {
    il = dzi_map(&mhi, hs, ht, n_rows, hidden, &s_view, &lay) &&
         make_map(&mw256, w, hidden, vocab, hidden, klg::BK, klg::DZI_BN / 2);
    if (!il && dzi_mode() == 2) return fail(KLG_ERR_CUDA, "interleaved-view tensor map rejected (KLG_DZI=2)");
  }
  if (!make_map(&mw_mn, w, hidden, vocab, hidden, 32, klg::BK, CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_map(&mhs_mn, hs, hidden, n_rows, hidden, 32, klg::BK, CU_TENSOR_MAP_SWIZZLE_64B))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  // fp32 outputs, written by TMA stores and reduce-adds
  alignas(64) CUtensorMap mdw, mdh;
  if ((d_w && !make_map(&mdw, d_w, hidden, vocab, hidden, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_DATA_TYPE_FLOAT32)) ||
      (d_hs && !make_map(&mdh, d_hs, hidden, n_rows, hidden, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed (outputs)");
  if (!d_w) mdw = mhs;   // unused placeholders
  if (!d_hs) mdh = mhs;
  // the exchange's TMA stores: one map per rank over its inbox [2 * world * rows_per_owner][H]
  alignas(64) klg::XrMaps xm{};
  if (xr && xr->tma)
    for (int p = 0; p < xr->world; ++p)
      if (!make_map(&xm.m[p], xr->inbox[p], hidden, (uint64_t)2 * xr->world * xr->rows_per_owner, hidden, 32, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32))
        return fail(KLG_ERR_CUDA, "tensor map (exchange inbox %d)", p);
  // The GEMMs store a tile's first addend and reduce-add the later ones: dH's first addend is
  // chunk 0's (plane 0's), a dW row's is its chunk's -- unless dW's K is split in two, whose
  // partial sums are reduce-added onto zero in either order.  So only dW of a shape with a K
  // split is zeroed (H % 8 == 0: a whole number of float4).
  bool dw_split = false;
  for (int64_t v0 = 0; d_w && !xr && v0 < vocab && !split; v0 += cols) {
    const int64_t wv = (vocab - v0) < cols ? (vocab - v0) : cols;
    if (pick_dw_split((int)n_rows, (int)wv, (int)hidden, bn) > 0) dw_split = true;
  }
  if (dw_split) {
    const long long n4 = vocab * hidden / 4;
    const int blocks = (int)std::min<long long>(cdiv(n4, 256), 4ll * num_sms());
    const int slot = trace_pre(s);
    cudaError_t ze = launch_k(klg::zero_f32x4_kernel, dim3(blocks), dim3(256), 0, s, 1, reinterpret_cast<float4*>(d_w), n4);
    trace_post(slot, s, KLG_KIND_ZERO);
    if (ze != cudaSuccess) return cuda_fail(ze, "launch zero_f32x4_kernel");
    ++g_launches;
  }

  klg::DualArgs a{};
  a.n_rows = (int)n_rows;
  a.n_rt = cdiv(n_rows, 256);   // pair tiles
  a.n_kb = cdiv(hidden, klg::BK);
  a.scale_log2 = inv_temp * 1.4426950408889634f;
  a.lse = lse;
  a.mask = mask;
  a.count = count;
  a.grad = grad;
  a.inv_temp = inv_temp;
  a.dz = dz;
  a.ld_dz = (int)ld_dz;
  a.a_parts = a_parts;
  int n_ap = 0;
  const int n_chunks = cdiv(vocab, cols);
  for (int64_t v0 = 0, ci = 0; v0 < vocab; v0 += cols, ++ci) {
    const int64_t wv = (vocab - v0) < cols ? (vocab - v0) : cols;
    if (tr) {
      klg::DztArgs t{};
      t.n_rows = (int)n_rows;
      t.v_begin = (int)v0;
      t.v_count = (int)wv;
      t.n_vp = cdiv(wv, 256);
      t.n_rt = cdiv(n_rows, klg::DZT_BN);
      const DztPlan P = plan_dzt(t.n_vp, t.n_rt, num_sms() / 2, n_rows, n_chunks);
      t.g = P.g;
      t.rpu = P.rpu;
      t.n_vg = P.n_vg;
      t.n_units = P.n_vg * P.n_rg;
      t.n_kb = cdiv(hidden, klg::BK);
      t.scale_log2 = inv_temp * 1.4426950408889634f;
      t.lse = lse;
      t.mask = mask;
      t.count = count;
      t.grad = grad;
      t.inv_temp = inv_temp;
      t.a_parts = a_parts;
      t.a_part_base = n_ap;
      n_ap += 2 * P.n_vg;   // one cross-term partial row per vocab group and CTA of the pair
      alignas(64) CUtensorMap mdzt_out;
      if (!make_map(&mdzt_out, dz, n_rows, wv, ld_n, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return fail(KLG_ERR_CUDA, "tensor map (dz^T store)");
      if ((rc = launch_dzt(mw, mhs, mht, mdzt_out, t, s))) return rc;
      if (d_hs || d_w) {
        // problem 0: dW chunk = dZ^T h_s (A = dZ^T, K-major); problem 1: dH += dZ W_chunk (A = dZ^T read MN-major)
        klg::PairGemmArgs g{};
        g.p[1] = gemm_problem(d_hs != nullptr, (int)n_rows, (int)hidden, (int)wv, bn, nullptr, (int)hidden,
                              v0 > 0 ? 1 : 0, 0, (int)v0, 1, 256, 0, 0);
        const int kb_split = pick_dw_split((int)n_rows, (int)wv, (int)hidden, bn);
        g.p[0] = gemm_problem(d_w != nullptr, (int)wv, (int)hidden, (int)n_rows, bn, nullptr, (int)hidden,
                              kb_split > 0 ? 1 : 0, 0, 0, 0, 256, kb_split, (int)v0);
        g.n_tiles = g.p[0].n_tiles + g.p[1].n_tiles;
        if (xr) g.xr = *xr;   // dW blocks go to their owners' inboxes (klg_xr.cuh)
        alignas(64) CUtensorMap mdzt_k, mdzt_mn;
        if (!make_map(&mdzt_k, dz, n_rows, wv, ld_n, klg::BK, klg::BM) ||
            !make_map(&mdzt_mn, dz, n_rows, wv, ld_n, 64, klg::BK))
          return fail(KLG_ERR_CUDA, "tensor map (dz^T operand)");
        if ((rc = launch_gemm_pair(bn, mdzt_k, mhs_mn, mdzt_mn, mw_mn, mdw, mdh, g, s, &xm))) return rc;
      }
      if (chunk_events && ci < n_events && chunk_events[ci]) {
        cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(chunk_events[ci]), s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord (chunk event)");
      }
      continue;
    }
    if (il) {
      klg::DziArgs b{};
      b.n_rows = (int)n_rows;
      b.v_begin = (int)v0;
      b.v_count = (int)wv;
      b.n_rt = cdiv(n_rows, klg::DZI_ROWS);
      b.n_vt = cdiv(wv, klg::DZI_BN);
      int n_uv;
      plan_dual(b.n_rt, b.n_vt, num_sms() / 2, b.vt_per_unit, n_uv, a_parts ? 8 : 64);
      b.n_units = b.n_rt * n_uv;
      b.n_kb = cdiv(hidden, klg::BK);
      b.s_view = s_view;
      b.scale_log2 = a.scale_log2;
      b.lse = lse;
      b.mask = mask;
      b.count = count;
      b.grad = grad;
      b.inv_temp = inv_temp;
      b.a_parts = a_parts;
      b.a_part_base = n_ap;
      n_ap += klg::DZI_CSPLIT * n_uv;   // one cross-term partial per unit and column half
      alignas(64) CUtensorMap mdz_out;
      if (!make_map(&mdz_out, dz, wv, n_rows, ld_dz, klg::DZI_STORE_COLS, 16))
        return fail(KLG_ERR_CUDA, "tensor map (dz store)");
      if ((rc = launch_dzi(lay, mhi, mw256, mdz_out, b, s))) return rc;
    } else {
      a.v_begin = (int)v0;
      a.v_count = (int)wv;
      a.n_vt = cdiv(wv, klg::DZP_BN);
      int n_uv;
      plan_dual(a.n_rt, a.n_vt, num_sms() / 2, a.vt_per_unit, n_uv, a_parts ? 8 : 64);
      a.n_units = a.n_rt * n_uv;
      a.a_part_base = n_ap;
      n_ap += klg::DZP_CSPLIT * n_uv;   // one cross-term partial per unit and column slice
      alignas(64) CUtensorMap mdz_out, mdz_out2;
      if (!make_map(&mdz_out, dz, wv, n_rows, ld_dz, klg::DZP_STORE_COLS, 32, CU_TENSOR_MAP_SWIZZLE_64B) ||
          (split && !make_map(&mdz_out2, dz + cols, wv, n_rows, ld_dz, klg::DZP_STORE_COLS, 32, CU_TENSOR_MAP_SWIZZLE_64B)))
        return fail(KLG_ERR_CUDA, "tensor map (dz store)");
      if (!split) mdz_out2 = mdz_out;
      if ((rc = launch_dual_pair<klg::MODE_DZ>(mhs, mht, mw, mdz_out, mdz_out2, a, s, split))) return rc;
    }
    if (!d_hs && !d_w) continue;
    // one grouped launch per dZ plane: problem 0 = dW chunk (longer tiles first), problem 1 = dH += dZ W_chunk
    // dW's K (all rows) may be split in two, at the point that gives the shortest
    // simulated schedule (the uneven pieces fill the gaps the equal tiles leave).  At most
    // two partial sums meet in any dW element, and the reduce-adds onto zero give the
    // same bits in either order, so dW stays deterministic.
    klg::PairGemmArgs g{};
    g.p[1] = gemm_problem(d_hs != nullptr, (int)n_rows, (int)hidden, (int)wv, bn, nullptr, (int)hidden, 1, 0,
                          (int)v0, 0, 256, 0, 0);
    const int kb_split = split ? 0 : pick_dw_split((int)n_rows, (int)wv, (int)hidden, bn);
    g.p[0] = gemm_problem(d_w != nullptr, (int)wv, (int)hidden, (int)n_rows, bn, nullptr, (int)hidden, 1, 0, 0, 1, 256,
                          kb_split, (int)v0);
    g.n_tiles = g.p[0].n_tiles + g.p[1].n_tiles;
    if (xr) g.xr = *xr;   // dW blocks go to their owners' inboxes (klg_xr.cuh)
    (void)ci;
    for (int plane = 0; plane < (split ? 2 : 1); ++plane) {
      g.p[1].accumulate = (v0 > 0 || plane > 0) ? 1 : 0;        // dH: store chunk 0's plane 0
      g.p[0].accumulate = (kb_split > 0 || plane > 0) ? 1 : 0;  // dW rows of this chunk: store plane 0
      const __nv_bfloat16* dzp = dz + plane * cols;
      alignas(64) CUtensorMap mdz_k, mdz_mn;
      if (!make_map(&mdz_k, dzp, wv, n_rows, ld_dz, klg::BK, klg::BM) ||
          !make_map(&mdz_mn, dzp, wv, n_rows, ld_dz, 64, klg::BK))
        return fail(KLG_ERR_CUDA, "tensor map (dz operand)");
      if ((rc = launch_gemm_pair(bn, mdz_mn, mhs_mn, mdz_k, mw_mn, mdw, mdh, g, s, &xm))) return rc;
    }
    if (chunk_events && ci < n_events && chunk_events[ci]) {
      cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(chunk_events[ci]), s);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord (chunk event)");
    }
  }
  if (n_ap_out) *n_ap_out = n_ap;
  return KLG_OK;
}

// Cross-term partial rows pass 2 writes for chunks of `cols` columns, at most: the transposed
// kernel's count when it runs, else the larger of the interleaved-view and row-major kernels'
// (which of the two runs depends on the input pointers; run_pass2 reports the rows written).
int pass2_parts(int64_t n_rows, int64_t hidden, int64_t vocab, int64_t cols, bool split = false) {
  int n_ap = 0;
  const int n_chunks = cdiv(vocab, cols);
  for (int64_t v0 = 0; v0 < vocab; v0 += cols) {
    const int64_t wv = (vocab - v0) < cols ? (vocab - v0) : cols;
    if (!split && dzt_on(hidden)) {
      n_ap += 2 * plan_dzt(cdiv(wv, 256), cdiv(n_rows, klg::DZT_BN), num_sms() / 2, n_rows, n_chunks).n_vg;
      continue;
    }
    int vpu, n_uv;
    plan_dual(cdiv(n_rows, 256), cdiv(wv, klg::DZP_BN), num_sms() / 2, vpu, n_uv, 8);
    int rows = klg::DZP_CSPLIT * n_uv;
    if (!split && dzi_on()) {
      plan_dual(cdiv(n_rows, klg::DZI_ROWS), cdiv(wv, klg::DZI_BN), num_sms() / 2, vpu, n_uv, 8);
      rows = std::max(rows, klg::DZI_CSPLIT * n_uv);
    }
    n_ap += rows;
  }
  return n_ap;
}

// Pass-1 partial records per row and view (lse_pair_kernel's units x column slices).
int pass1_parts(int64_t n_rows, int64_t vocab) {
  int vpu, n_uv;
  plan_dual(2 * cdiv(n_rows, 256), cdiv(vocab, klg::LSE_BN), num_sms() / 2, vpu, n_uv);
  return klg::LSE_CSPLIT * n_uv;
}

// Training-path workspace layout for a given total size: returns the dZ chunk width (or -1).
struct FwdBwdLayout {
  int64_t lse_parts_off, a_parts_off, dz_off, cols;
  int n_lp, n_ap;
};
int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }
FwdBwdLayout fwd_bwd_layout_uncached(int64_t n_rows, int64_t hidden, int64_t vocab, int64_t workspace_bytes,
                                     int planes) {
  FwdBwdLayout L{};
  L.n_lp = pass1_parts(n_rows, vocab);
  L.lse_parts_off = KLG_BWD_HEADER;
  L.a_parts_off = align256(L.lse_parts_off + (int64_t)L.n_lp * 2 * 2 * n_rows * 4);
  L.cols = -1;
  const int64_t full = (int64_t)cdiv(vocab, 128) * 128;
  // widest chunk that could fit (the cross-term partials only shrink the room), then narrower
  const int64_t dz_rows = round8(n_rows);   // dZ^T rows are padded to 16 bytes
  int64_t c = (workspace_bytes - L.a_parts_off) / (dz_rows * 2 * planes);
  c = std::min(full, (c / 128) * 128);
  for (; c >= 128; c -= 128) {
    if (cdiv(vocab, c) > KLG_BWD_HEADER / 4) break;
    const int n_ap = pass2_parts(n_rows, hidden, vocab, c, planes == 2);
    const int64_t dz_off = align256(L.a_parts_off + (int64_t)n_ap * n_rows * 4);
    if (dz_off + dz_rows * c * 2 * planes <= workspace_bytes) {
      L.cols = c;
      L.n_ap = n_ap;
      L.dz_off = dz_off;
      break;
    }
  }
  return L;
}

// Memoised: the layout is a pure function of the shape and workspace size.
FwdBwdLayout fwd_bwd_layout(int64_t n_rows, int64_t hidden, int64_t vocab, int64_t workspace_bytes, int planes = 1) {
  static std::mutex mu;
  static std::map<std::tuple<int64_t, int64_t, int64_t, int64_t, int, int>, FwdBwdLayout> memo;
  const auto key = std::make_tuple(n_rows, hidden, vocab, workspace_bytes, num_sms(), planes);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
  }
  const FwdBwdLayout L = fwd_bwd_layout_uncached(n_rows, hidden, vocab, workspace_bytes, planes);
  std::lock_guard<std::mutex> lk(mu);
  if (memo.size() > 256) memo.clear();
  memo[key] = L;
  return L;
}

// Pass 1 of the training path: both views' (m, S) per row over W's rows on CTA pairs
// (partial records into lse_parts, n_lp of them), merged into the log-sum-exps `lse` [2][N]
// and/or one merged record `rec` [2][2N].
int run_pass1(const void* hs, const void* ht, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab,
              float inv_temp, float* lse_parts, int n_lp, float* lse, float* rec, cudaStream_t s,
              const uint8_t* mask = nullptr, float* count = nullptr, unsigned* done = nullptr) {
  alignas(64) CUtensorMap mhs, mht, mw;
  if (!make_map(&mhs, hs, hidden, n_rows, hidden, klg::BK, klg::BM) ||
      !make_map(&mht, ht, hidden, n_rows, hidden, klg::BK, klg::BM) ||
      !make_map(&mw, w, hidden, vocab, hidden, klg::BK, klg::LSE_BN / 2))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  klg::LseArgs la{};
  la.n_rows = (int)n_rows;
  la.vocab = (int)vocab;
  la.n_rp = cdiv(n_rows, 256);
  la.n_vt = cdiv(vocab, klg::LSE_BN);
  plan_dual(2 * la.n_rp, la.n_vt, num_sms() / 2, la.vt_per_unit, la.n_uv);
  la.n_units = 2 * la.n_rp * la.n_uv;
  la.n_kb = cdiv(hidden, klg::BK);
  la.scale_log2 = inv_temp * 1.4426950408889634f;
  la.parts = lse_parts;
  la.n_views = 2;
  la.rep = 1;
  if (klg::LSE_CSPLIT * la.n_uv != n_lp) return fail(KLG_ERR_ARG, "internal plan mismatch");
  int rc = launch_lse_pair<klg::EPI_LSE>(mhs, mht, mw, la, s);
  if (rc) return rc;
  const int n2 = (int)(2 * n_rows);
  const int slot = trace_pre(s);
  const int extra = (count || done) ? 1 : 0;   // the block that counts the mask / clears *done
  cudaError_t e = launch_k(klg::lse_merge_kernel, dim3(cdiv(n2, 256) + extra), dim3(256), 0, s, 1, lse_parts, n_lp,
                           n2, lse, rec, mask, (int)n_rows, count, done);
  trace_post(slot, s, KLG_KIND_MERGE);
  if (e != cudaSuccess) return cuda_fail(e, "launch lse_merge_kernel");
  ++g_launches;
  return KLG_OK;
}

}  // namespace

extern "C" {

int klg_bwd(const void* hs, const void* ht, const void* w, const uint8_t* mask, const float* lse, const float* count,
            const float* grad, int64_t n_rows, int64_t hidden, int64_t vocab, float inv_temp, float* d_hs, float* d_w,
            void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !lse || !count) return fail(KLG_ERR_ARG, "null mask/lse/count");
  if (!d_hs && !d_w) return KLG_OK;
  if ((d_hs && !aligned16(d_hs)) || (d_w && !aligned16(d_w))) return fail(KLG_ERR_ALIGN, "outputs must be 16-byte aligned");
  const int64_t cols = klg_bwd_chunk_cols(n_rows, vocab, workspace_bytes);
  if (!workspace || cols < 0 || !aligned16(workspace))
    return fail(KLG_ERR_WORKSPACE, "backward workspace too small: needs >= %lld bytes",
                (long long)(KLG_BWD_HEADER + n_rows * 256));
  if ((rc = bind_device(hs))) return rc;
  NvtxRange nvtx_range("klg_bwd (pass 2)");

  __nv_bfloat16* dz = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + KLG_BWD_HEADER);
  return run_pass2(hs, ht, w, mask, lse, count, grad, n_rows, hidden, vocab, inv_temp, d_hs, d_w, dz, cols,
                   nullptr, nullptr, (cudaStream_t)stream);
}

}  // extern "C"

namespace {

// The exchange's stores from the dW GEMM: TMA tensor stores into the owners' inboxes (default),
// or 16-byte stores from registers with KLG_XR_TMA=0 (A/B timing).
bool xr_tma_on() {
  static const bool on = [] {
    const char* v = std::getenv("KLG_XR_TMA");
    return !(v && v[0] == '0');
  }();
  return on;
}

// The two kernels that finish the cross-rank dW exchange (klg_xr.cuh).  Their blocks wait only
// on other ranks' flags (block 0 publishes this rank's first), so a grid larger than what is
// resident at once cannot deadlock; four blocks per SM keep enough loads in flight.
int launch_xr(const klg::XrSync& x, cudaStream_t s) {
  int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::xr_reduce_kernel, dim3(4 * num_sms()), dim3(256), 0, s, 1, x);
  if (e == cudaSuccess) {
    ++g_launches;
    e = launch_k(klg::xr_wait_kernel, dim3(1), dim3(32), 0, s, 1, x);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launch xr_reduce_kernel / xr_wait_kernel");
  ++g_launches;
  // the gather on the copy engines: owner p's summed rows hold its 32-row blocks b = p, p + W,
  // ... back to back; each goes to rows 32 b of dW
  const size_t blk = (size_t)32 * x.hidden * 4;
  const int nb = cdiv(x.vocab, 32), tail = x.vocab - (nb - 1) * 32;   // rows of the last block
  for (int p = 0; p < x.world && p < nb; ++p) {
    const int own = (nb - 1 - p) / x.world + 1;                       // blocks of owner p
    const bool last_mine = (nb - 1) % x.world == p;
    const int full = own - ((last_mine && tail < 32) ? 1 : 0);
    const char* src = reinterpret_cast<const char*>(x.final_peer[p]);
    char* dst = reinterpret_cast<char*>(x.dw) + (size_t)p * blk;
    if (full > 0 && (e = cudaMemcpy2DAsync(dst, blk * x.world, src, blk, blk, full, cudaMemcpyDeviceToDevice, s)) !=
                        cudaSuccess)
      return cuda_fail(e, "dW gather copy");
    if (full < own &&
        (e = cudaMemcpyAsync(dst + (size_t)full * blk * x.world, src + (size_t)full * blk,
                             (size_t)tail * x.hidden * 4, cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
      return cuda_fail(e, "dW gather copy (last block)");
  }
  trace_post(slot, s, KLG_KIND_XR);
  return KLG_OK;
}

// Per-rank exchange buffer: [inbox world x 2 x rows_per_owner x H][final rows_per_owner x H] fp32,
// then the flags [2][XR_MAX_WORLD] u32 and the split records (256 bytes).
int64_t xr_rows_per_owner(int64_t vocab, int world) { return (int64_t)cdiv(cdiv(vocab, 32), world) * 32; }

klg::XrSync xr_sync(int64_t vocab, int64_t hidden, int world, int rank, void* const* bufs, uint32_t epoch, float* d_w) {
  klg::XrSync x{};
  x.world = world;
  x.rank = rank;
  x.rows_per_owner = (int)xr_rows_per_owner(vocab, world);
  x.hidden = (int)hidden;
  x.vocab = (int)vocab;
  x.epoch = epoch;
  const size_t inbox_f = (size_t)2 * world * x.rows_per_owner * hidden, final_f = (size_t)x.rows_per_owner * hidden;
  for (int p = 0; p < world; ++p) {
    float* base = static_cast<float*>(bufs[p]);
    x.inbox_peer[p] = base;
    x.final_peer[p] = base + inbox_f;
    x.flags_peer[p] = reinterpret_cast<uint32_t*>(base + inbox_f + final_f);
  }
  float* mine = static_cast<float*>(bufs[rank]);
  x.inbox = mine;
  x.final_rows = mine + inbox_f;
  x.flags = reinterpret_cast<uint32_t*>(mine + inbox_f + final_f);
  x.dw = d_w;
  return x;
}

// Workspace of the training step with `planes` bf16 planes of dZ (1, or 2 for the fp32-faithful path).
int64_t fwd_bwd_ws(int64_t n_rows, int64_t hidden, int64_t vocab, int planes) {
  if (n_rows < 1 || vocab < 1) return -1;
  const int64_t dz_bytes = klg_bwd_workspace_bytes(n_rows, hidden, vocab) - KLG_BWD_HEADER;
  const int64_t cols = dz_bytes / (round8(n_rows) * 2);
  FwdBwdLayout L = fwd_bwd_layout(n_rows, hidden, vocab, INT64_MAX / 4);
  const int n_ap = pass2_parts(n_rows, hidden, vocab, cols, planes == 2);
  return align256(L.a_parts_off + (int64_t)n_ap * n_rows * 4) + dz_bytes * planes;
}

// The training step on bf16 rows (validated, device bound): count, pass 1, pass 2, loss.
int fwd_bwd_core(const void* hs, const void* ht, const void* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
                 int64_t vocab, float inv_temp, int count_given, float* count, const float* grad, float* loss,
                 float* lse, float* row_kl, float* d_hs, float* d_w, void* workspace, int64_t workspace_bytes,
                 cudaStream_t s, int planes, void* const* chunk_events = nullptr, int n_events = 0,
                 const klg::XrSync* xs = nullptr) {
  int rc;
  const FwdBwdLayout L = fwd_bwd_layout(n_rows, hidden, vocab, workspace_bytes, planes);
  if (L.cols < 0)
    return fail(KLG_ERR_WORKSPACE, "workspace of %lld bytes too small (see the *_workspace_bytes functions)",
                (long long)workspace_bytes);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* lse_parts = reinterpret_cast<float*>(ws + L.lse_parts_off);
  float* a_parts = reinterpret_cast<float*>(ws + L.a_parts_off);
  unsigned* done = reinterpret_cast<unsigned*>(ws);   // first word of the reserved header: the loss kernel's counter

  // pass 1: log-sum-exp of both views on CTA pairs; the merge launch also counts the mask
  // (unless the caller gives the count) and clears the loss kernel's completion counter
  if ((rc = run_pass1(hs, ht, w, n_rows, hidden, vocab, inv_temp, lse_parts, L.n_lp, lse, nullptr, s, mask,
                      count_given ? nullptr : count, done)))
    return rc;
  // pass 2: dZ chunks (+ KL cross-term partials) and the dW / dH GEMMs
  int n_ap = 0;
  __nv_bfloat16* dz = reinterpret_cast<__nv_bfloat16*>(ws + L.dz_off);
  klg::XrArgs xa{};
  if (xs) {
    xa.world = xs->world;
    xa.rank = xs->rank;
    xa.rows_per_owner = xs->rows_per_owner;
    xa.tma = xr_tma_on() ? 1 : 0;
    for (int p = 0; p < xs->world; ++p) xa.inbox[p] = xs->inbox_peer[p];
  }
  if ((rc = run_pass2(hs, ht, w, mask, lse, count, grad, n_rows, hidden, vocab, inv_temp, d_hs, d_w, dz,
                      L.cols, a_parts, &n_ap, s, planes == 2, chunk_events, n_events, xs ? &xa : nullptr)))
    return rc;
  if (n_ap > L.n_ap) return fail(KLG_ERR_ARG, "internal plan mismatch (cross-term partials)");
  // per-row KL in 256-row blocks (block sums reuse the pass-1 partial area); the last block
  // to finish forms the loss
  const int nb = cdiv(n_rows, 256);
  float* block_sums = lse_parts;
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::row_kl_pair_kernel, dim3(nb), dim3(256), 0, s, 1, lse, a_parts, n_ap, mask,
                           (int)n_rows, row_kl, block_sums, static_cast<const float*>(count), loss, done);
  trace_post(slot, s, KLG_KIND_FINALIZE);
  if (e != cudaSuccess) return cuda_fail(e, "launch row_kl_pair_kernel");
  ++g_launches;
  if (xs) return launch_xr(*xs, s);
  return KLG_OK;
}

// fp32-faithful inputs: [hi | hi | lo] rows for the hidden states, [hi | lo | hi] for the lm_head.
int launch_split3(const float* x, int64_t n_rows, int64_t hidden, int order, __nv_bfloat16* out, cudaStream_t s) {
  const long long n = n_rows * hidden;
  const int blocks = (int)std::min<long long>(cdiv(n, 256), 8ll * num_sms());
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::split3_kernel, dim3(blocks), dim3(256), 0, s, 1, x, (long long)n_rows, (int)hidden,
                           order, out);
  trace_post(slot, s, KLG_KIND_CAST);
  if (e != cudaSuccess) return cuda_fail(e, "launch split3_kernel");
  ++g_launches;
  return KLG_OK;
}

int launch_fold2(const float* in, int64_t n_rows, int64_t hidden, int a, int b, float* out, cudaStream_t s) {
  const long long n = n_rows * hidden;
  const int blocks = (int)std::min<long long>(cdiv(n, 256), 8ll * num_sms());
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::fold2_kernel, dim3(blocks), dim3(256), 0, s, 1, in, (long long)n_rows, (int)hidden,
                           a, b, out);
  trace_post(slot, s, KLG_KIND_CAST);
  if (e != cudaSuccess) return cuda_fail(e, "launch fold2_kernel");
  ++g_launches;
  return KLG_OK;
}

// Layout of the fp32 path's workspace: split rows, then (fwd_bwd) the 3H-wide gradients, then
// the bf16 path's own workspace.
struct F32Layout {
  int64_t hs, ht, w, dh, dw, core, total;
};
F32Layout f32_layout(int64_t n_rows, int64_t hidden, int64_t vocab, int64_t core_bytes, bool grads) {
  F32Layout L{};
  const int64_t h3 = 3 * hidden;
  L.hs = 0;
  L.ht = align256(L.hs + n_rows * h3 * 2);
  L.w = align256(L.ht + n_rows * h3 * 2);
  L.dh = align256(L.w + vocab * h3 * 2);
  L.dw = align256(L.dh + (grads ? n_rows * h3 * 4 : 0));
  L.core = align256(L.dw + (grads ? vocab * h3 * 4 : 0));
  L.total = core_bytes < 0 ? -1 : L.core + core_bytes;
  return L;
}

int check_f32(const float* hs, const float* ht, const float* w, int64_t n_rows, int64_t hidden, int64_t vocab,
              float inv_temp) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (3 * hidden > (1ll << 20)) return fail(KLG_ERR_ARG, "hidden=%lld too large for the fp32 path", (long long)hidden);
  return KLG_OK;
}

}  // namespace

extern "C" {

int64_t klg_fwd_bwd_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab) {
  return fwd_bwd_ws(n_rows, hidden, vocab, 1);
}

int64_t klg_fwd_bwd_chunk_cols(int64_t n_rows, int64_t hidden, int64_t vocab, int64_t workspace_bytes) {
  if (n_rows < 1 || vocab < 1 || hidden < 8) return -1;
  return fwd_bwd_layout(n_rows, hidden, vocab, workspace_bytes).cols;
}

int klg_fwd_bwd(const void* hs, const void* ht, const void* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
                int64_t vocab, float inv_temp, int count_given, float* count, const float* grad, float* loss,
                float* lse, float* row_kl, float* d_hs, float* d_w, void* workspace, int64_t workspace_bytes,
                void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !count || !loss || !lse) return fail(KLG_ERR_ARG, "null mask/count/loss/lse");
  if ((d_hs && !aligned16(d_hs)) || (d_w && !aligned16(d_w))) return fail(KLG_ERR_ALIGN, "outputs must be 16-byte aligned");
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if ((rc = bind_device(hs))) return rc;   // the layout depends on the SM count of hs's device
  NvtxRange nvtx_range("klg_fwd_bwd");
  return fwd_bwd_core(hs, ht, w, mask, n_rows, hidden, vocab, inv_temp, count_given, count, grad, loss, lse, row_kl,
                      d_hs, d_w, workspace, workspace_bytes, (cudaStream_t)stream, 1);
}

int klg_fwd_bwd_events(const void* hs, const void* ht, const void* w, const uint8_t* mask, int64_t n_rows,
                       int64_t hidden, int64_t vocab, float inv_temp, int count_given, float* count, const float* grad,
                       float* loss, float* lse, float* row_kl, float* d_hs, float* d_w, void* workspace,
                       int64_t workspace_bytes, void* const* chunk_events, int n_events, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !count || !loss || !lse) return fail(KLG_ERR_ARG, "null mask/count/loss/lse");
  if ((d_hs && !aligned16(d_hs)) || (d_w && !aligned16(d_w))) return fail(KLG_ERR_ALIGN, "outputs must be 16-byte aligned");
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if (n_events < 0 || (n_events > 0 && !chunk_events)) return fail(KLG_ERR_ARG, "bad chunk event array");
  if ((rc = bind_device(hs))) return rc;
  const int64_t cols = fwd_bwd_layout(n_rows, hidden, vocab, workspace_bytes).cols;
  if (cols > 0 && n_events < cdiv(vocab, cols))
    return fail(KLG_ERR_ARG, "%d chunk events for %d chunks (klg_fwd_bwd_chunk_cols gives the chunk width)", n_events,
                cdiv(vocab, cols));
  NvtxRange nvtx_range("klg_fwd_bwd_events");
  return fwd_bwd_core(hs, ht, w, mask, n_rows, hidden, vocab, inv_temp, count_given, count, grad, loss, lse, row_kl,
                      d_hs, d_w, workspace, workspace_bytes, (cudaStream_t)stream, 1, chunk_events, n_events);
}

int64_t klg_xr_buffer_bytes(int64_t vocab, int64_t hidden, int world) {
  if (vocab < 1 || hidden < 8 || hidden % 8 != 0 || world < 2 || world > klg::XR_MAX_WORLD) return -1;
  const int64_t rpo = xr_rows_per_owner(vocab, world);
  return ((int64_t)2 * world + 1) * rpo * hidden * 4 + 256;   // flags and split records: 192 of 256 bytes
}

int klg_fwd_bwd_xr(const void* hs, const void* ht, const void* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
                   int64_t vocab, float inv_temp, int count_given, float* count, const float* grad, float* loss,
                   float* lse, float* row_kl, float* d_hs, float* d_w, void* workspace, int64_t workspace_bytes,
                   int world, int rank, void* const* peer_buffers, uint32_t epoch, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !count || !loss || !lse || !d_w) return fail(KLG_ERR_ARG, "null mask/count/loss/lse/d_w");
  if (world < 2 || world > klg::XR_MAX_WORLD || rank < 0 || rank >= world || !peer_buffers)
    return fail(KLG_ERR_ARG, "world %d / rank %d out of range or no peer buffers", world, rank);
  for (int p = 0; p < world; ++p)
    if (!peer_buffers[p] || !aligned16(peer_buffers[p])) return fail(KLG_ERR_ALIGN, "peer buffer %d null or misaligned", p);
  if ((d_hs && !aligned16(d_hs)) || !aligned16(d_w)) return fail(KLG_ERR_ALIGN, "outputs must be 16-byte aligned");
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if ((rc = bind_device(hs))) return rc;
  NvtxRange nvtx_range("klg_fwd_bwd_xr");
  klg::XrSync xs = xr_sync(vocab, hidden, world, rank, peer_buffers, epoch, d_w);
  // which chunks split dW's K (the GEMM's plan): their rows carry a second half in slot 1
  const FwdBwdLayout L = fwd_bwd_layout(n_rows, hidden, vocab, workspace_bytes);
  if (L.cols > 0) {
    const int bn = gemm_bn(hidden);
    const int64_t last_start = (int64_t)(cdiv(vocab, L.cols) - 1) * L.cols;
    xs.cols = (int)L.cols;
    xs.last_start = (int)last_start;
    xs.split_full = pick_dw_split((int)n_rows, (int)L.cols, (int)hidden, bn) > 0;
    xs.split_last = pick_dw_split((int)n_rows, (int)(vocab - last_start), (int)hidden, bn) > 0;
  }
  return fwd_bwd_core(hs, ht, w, mask, n_rows, hidden, vocab, inv_temp, count_given, count, grad, loss, lse, row_kl,
                      d_hs, d_w, workspace, workspace_bytes, (cudaStream_t)stream, 1, nullptr, 0, &xs);
}

int klg_xr_alloc(int device, int64_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes < 1) return fail(KLG_ERR_ARG, "bad arguments to klg_xr_alloc");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice (klg_xr_alloc)");
  void* p = nullptr;
  if ((e = cudaMalloc(&p, (size_t)bytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc (exchange buffer)");
  if ((e = cudaMemset(p, 0, (size_t)bytes)) != cudaSuccess ||
      (e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p)) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "exchange buffer set-up");
  }
  *ptr = p;
  return KLG_OK;
}

int klg_xr_open(int device, const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(KLG_ERR_ARG, "bad arguments to klg_xr_open");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice (klg_xr_open)");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  if ((e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
    return cuda_fail(e, "cudaIpcOpenMemHandle (peer exchange buffer)");
  return KLG_OK;
}

int klg_xr_close(void* ptr, int own) {
  if (!ptr) return KLG_OK;
  cudaError_t e = own ? cudaFree(ptr) : cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? KLG_OK : cuda_fail(e, "exchange buffer release");
}

int klg_selftest_xr_timeout(void* buffer, int64_t vocab, int64_t hidden, void* stream) {
  if (!buffer || !aligned16(buffer) || klg_xr_buffer_bytes(vocab, hidden, 2) < 0)
    return fail(KLG_ERR_ARG, "bad arguments to klg_selftest_xr_timeout");
  if (int rc = bind_device(buffer)) return rc;
  void* bufs[2] = {buffer, buffer};
  klg::XrSync x = xr_sync(vocab, hidden, 2, 0, bufs, 1u, nullptr);
  x.stall = 1;
  cudaError_t e = launch_k(klg::xr_reduce_kernel, dim3(1), dim3(256), 0, (cudaStream_t)stream, 1, x);
  if (e != cudaSuccess) return cuda_fail(e, "launch xr_reduce_kernel (self-test)");
  ++g_launches;
  return KLG_OK;
}

// ---------------------------------------------------------------- fp32-faithful path
int64_t klg_fwd_bwd_f32_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab) {
  if (n_rows < 1 || vocab < 1 || hidden < 8) return -1;
  return f32_layout(n_rows, hidden, vocab, fwd_bwd_ws(n_rows, 3 * hidden, vocab, 2), true).total;
}

int klg_fwd_bwd_f32(const float* hs, const float* ht, const float* w, const uint8_t* mask, int64_t n_rows,
                    int64_t hidden, int64_t vocab, float inv_temp, int count_given, float* count, const float* grad,
                    float* loss, float* lse, float* row_kl, float* d_hs, float* d_w, void* workspace,
                    int64_t workspace_bytes, void* stream) {
  int rc = check_f32(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !count || !loss || !lse) return fail(KLG_ERR_ARG, "null mask/count/loss/lse");
  if ((d_hs && !aligned16(d_hs)) || (d_w && !aligned16(d_w))) return fail(KLG_ERR_ALIGN, "outputs must be 16-byte aligned");
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if ((rc = bind_device(hs))) return rc;
  const F32Layout F = f32_layout(n_rows, hidden, vocab, 0, true);
  if (workspace_bytes <= F.core)
    return fail(KLG_ERR_WORKSPACE, "fp32 workspace of %lld bytes too small (see klg_fwd_bwd_f32_workspace_bytes)",
                (long long)workspace_bytes);
  NvtxRange nvtx_range("klg_fwd_bwd_f32");
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto* hs3 = reinterpret_cast<__nv_bfloat16*>(ws + F.hs);
  auto* ht3 = reinterpret_cast<__nv_bfloat16*>(ws + F.ht);
  auto* w3 = reinterpret_cast<__nv_bfloat16*>(ws + F.w);
  float* dh3 = d_hs ? reinterpret_cast<float*>(ws + F.dh) : nullptr;
  float* dw3 = d_w ? reinterpret_cast<float*>(ws + F.dw) : nullptr;
  if ((rc = launch_split3(hs, n_rows, hidden, 0, hs3, s)) || (rc = launch_split3(ht, n_rows, hidden, 0, ht3, s)) ||
      (rc = launch_split3(w, vocab, hidden, 1, w3, s)))
    return rc;
  if ((rc = fwd_bwd_core(hs3, ht3, w3, mask, n_rows, 3 * hidden, vocab, inv_temp, count_given, count, grad, loss, lse,
                         row_kl, dh3, dw3, ws + F.core, workspace_bytes - F.core, s, 2)))
    return rc;
  // dH' = dZ [W_hi | W_lo | W_hi] -> dH = blocks 0 + 1;  dW' = dZ^T [h_hi | h_hi | h_lo] -> dW = blocks 0 + 2
  if (d_hs && (rc = launch_fold2(dh3, n_rows, hidden, 0, 1, d_hs, s))) return rc;
  if (d_w && (rc = launch_fold2(dw3, vocab, hidden, 0, 2, d_w, s))) return rc;
  return KLG_OK;
}

int64_t klg_fwd_f32_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab) {
  if (n_rows < 1 || vocab < 1 || hidden < 8) return -1;
  return f32_layout(n_rows, hidden, vocab, klg_fwd_workspace_bytes(n_rows, vocab), false).total;
}

int klg_fwd_f32(const float* hs, const float* ht, const float* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
                int64_t vocab, float inv_temp, int count_given, float* count, float* loss, float* lse, float* row_kl,
                void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_f32(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !count || !loss || !lse) return fail(KLG_ERR_ARG, "null output pointer");
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if ((rc = bind_device(hs))) return rc;
  const F32Layout F = f32_layout(n_rows, hidden, vocab, 0, false);
  if (workspace_bytes <= F.core)
    return fail(KLG_ERR_WORKSPACE, "fp32 workspace of %lld bytes too small (see klg_fwd_f32_workspace_bytes)",
                (long long)workspace_bytes);
  NvtxRange nvtx_range("klg_fwd_f32");
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto* hs3 = reinterpret_cast<__nv_bfloat16*>(ws + F.hs);
  auto* ht3 = reinterpret_cast<__nv_bfloat16*>(ws + F.ht);
  auto* w3 = reinterpret_cast<__nv_bfloat16*>(ws + F.w);
  if ((rc = launch_split3(hs, n_rows, hidden, 0, hs3, s)) || (rc = launch_split3(ht, n_rows, hidden, 0, ht3, s)) ||
      (rc = launch_split3(w, vocab, hidden, 1, w3, s)))
    return rc;
  return klg_fwd(hs3, ht3, w3, mask, n_rows, 3 * hidden, vocab, inv_temp, count_given, count, loss, lse, row_kl,
                 ws + F.core, workspace_bytes - F.core, stream);
}

// ---------------------------------------------------------------- training step in pieces (vocab sharding)
int64_t klg_lse_workspace_bytes(int64_t n_rows, int64_t vocab) {
  if (n_rows < 1 || vocab < 1 || n_rows > (1ll << 30) || vocab > (1ll << 30)) return -1;
  return (int64_t)pass1_parts(n_rows, vocab) * 2 * 2 * n_rows * 4;
}

int klg_lse_record(const void* hs, const void* ht, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab,
                   float inv_temp, float* rec, void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!rec || !aligned16(rec)) return fail(KLG_ERR_ARG, "rec must be non-null and 16-byte aligned");
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if ((rc = bind_device(hs))) return rc;   // the plan depends on the SM count of hs's device
  const int n_lp = pass1_parts(n_rows, vocab);
  const int64_t need = (int64_t)n_lp * 2 * 2 * n_rows * 4;
  if (workspace_bytes < need)
    return fail(KLG_ERR_WORKSPACE, "pass-1 workspace needs %lld bytes (see klg_lse_workspace_bytes)", (long long)need);
  NvtxRange nvtx_range("klg_lse_record");
  return run_pass1(hs, ht, w, n_rows, hidden, vocab, inv_temp, static_cast<float*>(workspace), n_lp, nullptr, rec,
                   (cudaStream_t)stream);
}

int klg_lse_merge(const float* recs, int n_rec, int64_t n_rows, float* lse, void* stream) {
  if (!recs || !lse || n_rec < 1 || n_rows < 1 || n_rows > (1ll << 29)) return fail(KLG_ERR_ARG, "bad arguments to klg_lse_merge");
  if (int rc = bind_device(recs)) return rc;
  const int n2 = (int)(2 * n_rows);
  cudaStream_t s = (cudaStream_t)stream;
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::lse_merge_kernel, dim3(cdiv(n2, 256)), dim3(256), 0, s, 1, recs, n_rec, n2, lse,
                           static_cast<float*>(nullptr), static_cast<const uint8_t*>(nullptr), 0,
                           static_cast<float*>(nullptr), static_cast<unsigned*>(nullptr));
  trace_post(slot, s, KLG_KIND_MERGE);
  if (e != cudaSuccess) return cuda_fail(e, "launch lse_merge_kernel");
  ++g_launches;
  return KLG_OK;
}

int64_t klg_pass2_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab) {
  return klg_fwd_bwd_workspace_bytes(n_rows, hidden, vocab);
}

int klg_pass2(const void* hs, const void* ht, const void* w, const uint8_t* mask, const float* lse, const float* count,
              const float* grad, int64_t n_rows, int64_t hidden, int64_t vocab, float inv_temp, float* d_hs, float* d_w,
              float* cross, void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !lse || !count || !cross) return fail(KLG_ERR_ARG, "null mask/lse/count/cross");
  if ((d_hs && !aligned16(d_hs)) || (d_w && !aligned16(d_w))) return fail(KLG_ERR_ALIGN, "outputs must be 16-byte aligned");
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if ((rc = bind_device(hs))) return rc;   // the layout depends on the SM count of hs's device
  const FwdBwdLayout L = fwd_bwd_layout(n_rows, hidden, vocab, workspace_bytes);
  if (L.cols < 0)
    return fail(KLG_ERR_WORKSPACE, "workspace of %lld bytes too small (see klg_pass2_workspace_bytes)",
                (long long)workspace_bytes);
  NvtxRange nvtx_range("klg_pass2");
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* a_parts = reinterpret_cast<float*>(ws + L.a_parts_off);
  __nv_bfloat16* dz = reinterpret_cast<__nv_bfloat16*>(ws + L.dz_off);
  int n_ap = 0;
  if ((rc = run_pass2(hs, ht, w, mask, lse, count, grad, n_rows, hidden, vocab, inv_temp, d_hs, d_w, dz, L.cols,
                      a_parts, &n_ap, s)))
    return rc;
  if (n_ap > L.n_ap) return fail(KLG_ERR_ARG, "internal plan mismatch (cross-term partials)");
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::cross_sum_kernel, dim3(cdiv(n_rows, 256)), dim3(256), 0, s, 1, a_parts, n_ap,
                           (int)n_rows, cross);
  trace_post(slot, s, KLG_KIND_FINALIZE);
  if (e != cudaSuccess) return cuda_fail(e, "launch cross_sum_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_kl_loss(const float* lse, const float* cross, const uint8_t* mask, int64_t n_rows, const float* count,
                float* loss, float* row_kl, void* stream) {
  if (!lse || !cross || !mask || !count || !loss || n_rows < 1 || n_rows > (1ll << 30))
    return fail(KLG_ERR_ARG, "bad arguments to klg_kl_loss");
  if (int rc = bind_device(lse)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::kl_loss_kernel, dim3(1), dim3(1024), 0, s, 1, lse, cross, mask, (int)n_rows, count,
                           loss, row_kl);
  trace_post(slot, s, KLG_KIND_FINALIZE);
  if (e != cudaSuccess) return cuda_fail(e, "launch kl_loss_kernel");
  ++g_launches;
  return KLG_OK;
}

// ---------------------------------------------------------------- lm_head sampling (inference)
namespace {
int sample_plan(int64_t n_rows, int64_t vocab, klg::LseArgs& la) {
  la.n_rows = (int)n_rows;
  la.vocab = (int)vocab;
  la.n_rp = cdiv(n_rows, 256);
  la.n_vt = cdiv(vocab, klg::LSE_BN);
  la.n_views = 1;
  la.rep = n_rows <= 64 ? 4 : n_rows <= 128 ? 2 : 1;
  // few row tiles (decode) spread the vocab over more CTA pairs: units of >= 2 tiles
  plan_dual(la.n_rp, la.n_vt, num_sms() / 2, la.vt_per_unit, la.n_uv, num_sms() / 2, 2);
  la.n_units = la.n_rp * la.n_uv;
  return klg::LSE_CSPLIT * la.rep * la.n_uv;
}

// Record groups of the first merge launch: one when the rows alone give the GPU enough
// blocks, else groups of ~32 records (two per warp) merged again by a second launch.
int sample_merge_groups(int64_t n_rows, int n_part) {
#ifndef KLG_SMERGE_SINGLE
#define KLG_SMERGE_SINGLE 64
#endif
  if (cdiv(n_rows, 32) >= num_sms() || n_part <= KLG_SMERGE_SINGLE) return 1;
  const int g = cdiv(n_part, 32);
  return g < 64 ? g : 64;
}

int64_t sample_workspace(int64_t n_rows, int n_part) {
  const int g = sample_merge_groups(n_rows, n_part);
  return ((int64_t)n_part + (g > 1 ? g : 0)) * 5 * n_rows * 4;
}
}  // namespace

int64_t klg_lm_head_sample_workspace_bytes(int64_t n_rows, int64_t vocab) {
  if (n_rows < 1 || vocab < 1 || n_rows > (1ll << 30) || vocab > (1ll << 30)) return -1;
  klg::LseArgs la{};
  return sample_workspace(n_rows, sample_plan(n_rows, vocab, la));
}

int klg_lm_head_sample(const void* h, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab, float inv_temp,
                       int sample, uint64_t seed, int32_t* tokens, float* logit, float* lse, void* workspace,
                       int64_t workspace_bytes, void* stream) {
  int rc = check_problem(h, h, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!tokens || !logit || !lse) return fail(KLG_ERR_ARG, "null output pointer");
  // at least one record per row and epilogue column slice: checked before any device call
  if (!workspace || workspace_bytes < (int64_t)klg::LSE_CSPLIT * 5 * n_rows * 4 || !aligned16(workspace))
    return fail(KLG_ERR_WORKSPACE, "sampling workspace needs at least %lld bytes (16-byte aligned)",
                (long long)klg::LSE_CSPLIT * 5 * n_rows * 4);
  if ((rc = bind_device(h))) return rc;   // the plan depends on the SM count of h's device
  klg::LseArgs la{};
  const int n_part = sample_plan(n_rows, vocab, la);
  const int64_t need = sample_workspace(n_rows, n_part);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(KLG_ERR_WORKSPACE, "sampling workspace needs %lld bytes (16-byte aligned)", (long long)need);
  NvtxRange nvtx_range("klg_lm_head_sample");
  cudaStream_t s = (cudaStream_t)stream;
  la.n_kb = cdiv(hidden, klg::BK);
  la.scale_log2 = inv_temp * 1.4426950408889634f;
  la.parts = static_cast<float*>(workspace);
  la.seed_lo = (uint32_t)seed;
  la.seed_hi = (uint32_t)(seed >> 32);
  alignas(64) CUtensorMap mh, mh64, mw;   // mh64: box of 64 rows for the 4-copy row replication
  if (!make_map(&mh, h, hidden, n_rows, hidden, klg::BK, klg::BM) ||
      !make_map(&mh64, h, hidden, n_rows, hidden, klg::BK, 64) ||
      !make_map(&mw, w, hidden, vocab, hidden, klg::BK, klg::LSE_BN / 2))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  rc = sample ? launch_lse_pair<klg::EPI_SAMPLE>(mh, mh64, mw, la, s) : launch_lse_pair<klg::EPI_GREEDY>(mh, mh64, mw, la, s);
  if (rc) return rc;
  const int groups = sample_merge_groups(n_rows, n_part);
  const float* parts = static_cast<const float*>(workspace);
  float* grouped = static_cast<float*>(workspace) + (size_t)n_part * 5 * n_rows;
  for (int pass = groups > 1 ? 0 : 1; pass < 2; ++pass) {
    const int slot = trace_pre(s);
    cudaError_t e = pass == 0
        ? launch_k(klg::sample_merge_kernel, dim3(cdiv(n_rows, 32), groups), dim3(32 * klg::SMERGE_WARPS), 0, s, 1,
                   parts, n_part, (int)n_rows, grouped, tokens, logit, lse)
        : launch_k(klg::sample_merge_kernel, dim3(cdiv(n_rows, 32), 1), dim3(32 * klg::SMERGE_WARPS), 0, s, 1,
                   groups > 1 ? static_cast<const float*>(grouped) : parts, groups > 1 ? groups : n_part,
                   (int)n_rows, static_cast<float*>(nullptr), tokens, logit, lse);
    trace_post(slot, s, KLG_KIND_MERGE);
    if (e != cudaSuccess) return cuda_fail(e, "launch sample_merge_kernel");
    ++g_launches;
  }
  return KLG_OK;
}

// ---------------------------------------------------------------- filtered sampling (top-k / top-p)
namespace {
struct FilterLayout {
  int64_t rec, cmax, thr, lse, tok, lgt, cnt, cz, ci, total;
};
FilterLayout filter_layout(int64_t n_rows, int64_t vocab, int64_t cap, int n_part) {
  FilterLayout L{};
  const int64_t n_ck = cdiv(vocab, 32);
  L.rec = 0;
  L.cmax = align256(L.rec + sample_workspace(n_rows, n_part));
  L.thr = align256(L.cmax + n_rows * n_ck * 4);
  L.lse = align256(L.thr + n_rows * 4);
  L.tok = align256(L.lse + n_rows * 4);
  L.lgt = align256(L.tok + n_rows * 4);
  L.cnt = align256(L.lgt + n_rows * 4);
  L.cz = align256(L.cnt + n_rows * 4);
  L.ci = align256(L.cz + n_rows * cap * 4);
  L.total = align256(L.ci + n_rows * cap * 4);
  return L;
}
}  // namespace

int64_t klg_lm_head_sample_filtered_workspace_bytes(int64_t n_rows, int64_t vocab, int64_t cap) {
  if (n_rows < 1 || vocab < 1 || n_rows > (1ll << 24) || vocab > (1ll << 24) || cap < 1 || cap > vocab) return -1;
  klg::LseArgs la{};
  return filter_layout(n_rows, vocab, cap, sample_plan(n_rows, vocab, la)).total;
}

int klg_lm_head_sample_filtered(const void* h, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab,
                                float inv_temp, int top_k, float top_p, uint64_t seed, int64_t cap, int32_t* tokens,
                                float* logit, float* lse, int* overflow, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  int rc = check_problem(h, h, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!tokens || !logit || !lse || !overflow) return fail(KLG_ERR_ARG, "null output pointer");
  if (top_k < 0 || !(top_p > 0.f) || top_p > 1.f) return fail(KLG_ERR_ARG, "top_k must be >= 0 and top_p in (0, 1]");
  if (n_rows > (1ll << 24) || vocab > (1ll << 24) || cap < 1 || cap > vocab)
    return fail(KLG_ERR_ARG, "bad filtered-sampling shape N=%lld V=%lld cap=%lld", (long long)n_rows, (long long)vocab,
                (long long)cap);
  if (!workspace || !aligned16(workspace)) return fail(KLG_ERR_WORKSPACE, "null or misaligned workspace");
  if ((rc = bind_device(h))) return rc;
  klg::LseArgs la{};
  const int n_part = sample_plan(n_rows, vocab, la);
  const FilterLayout F = filter_layout(n_rows, vocab, cap, n_part);
  if (workspace_bytes < F.total)
    return fail(KLG_ERR_WORKSPACE, "filtered-sampling workspace needs %lld bytes", (long long)F.total);
  NvtxRange nvtx_range("klg_lm_head_sample_filtered");
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* rec = reinterpret_cast<float*>(ws + F.rec);
  float* cmax = reinterpret_cast<float*>(ws + F.cmax);
  float* thr = reinterpret_cast<float*>(ws + F.thr);
  float* lse_all = reinterpret_cast<float*>(ws + F.lse);
  int32_t* tok_a = reinterpret_cast<int32_t*>(ws + F.tok);
  float* lgt_a = reinterpret_cast<float*>(ws + F.lgt);
  int* cnt = reinterpret_cast<int*>(ws + F.cnt);
  float* cz = reinterpret_cast<float*>(ws + F.cz);
  int* ci = reinterpret_cast<int*>(ws + F.ci);
  la.n_kb = cdiv(hidden, klg::BK);
  la.scale_log2 = inv_temp * 1.4426950408889634f;
  la.parts = rec;
  la.n_ck = cdiv(vocab, 32);
  la.cap = (int)cap;
  alignas(64) CUtensorMap mh, mh64, mw;
  if (!make_map(&mh, h, hidden, n_rows, hidden, klg::BK, klg::BM) ||
      !make_map(&mh64, h, hidden, n_rows, hidden, klg::BK, 64) ||
      !make_map(&mw, w, hidden, vocab, hidden, klg::BK, klg::LSE_BN / 2))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  // sweep 1: per row (m, S) of z / T and the 32-column chunk maxima; merged to the row's lse
  la.cmax = cmax;
  if ((rc = launch_lse_pair<klg::EPI_GREEDY>(mh, mh64, mw, la, s))) return rc;
  {
    const int slot = trace_pre(s);
    cudaError_t e = launch_k(klg::sample_merge_kernel, dim3(cdiv(n_rows, 32), 1), dim3(32 * klg::SMERGE_WARPS), 0, s, 1,
                             static_cast<const float*>(rec), n_part, (int)n_rows, static_cast<float*>(nullptr), tok_a,
                             lgt_a, lse_all);
    trace_post(slot, s, KLG_KIND_MERGE);
    if (e != cudaSuccess) return cuda_fail(e, "launch sample_merge_kernel");
    ++g_launches;
  }
  // per row: the threshold no surviving logit is below
  {
    const int slot = trace_pre(s);
    cudaError_t e = launch_k(klg::filter_threshold_kernel, dim3((unsigned)n_rows), dim3(klg::FILT_THREADS), 0, s, 1,
                             static_cast<const float*>(cmax), la.n_ck, static_cast<const float*>(lse_all), inv_temp,
                             top_k, top_p, thr);
    trace_post(slot, s, KLG_KIND_SAMPLE);
    if (e != cudaSuccess) return cuda_fail(e, "launch filter_threshold_kernel");
    ++g_launches;
  }
  // sweep 2: the candidates (every logit at or above the threshold)
  cudaError_t e = cudaMemsetAsync(cnt, 0, (size_t)n_rows * sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync (candidate counters)");
  e = cudaMemsetAsync(overflow, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync (overflow flag)");
  la.cmax = nullptr;
  la.thr = thr;
  la.cand_cnt = cnt;
  la.cand_z = cz;
  la.cand_i = ci;
  if ((rc = launch_lse_pair<klg::EPI_CAND>(mh, mh64, mw, la, s))) return rc;
  // per row: top-k / top-p on the candidates and the Gumbel-max draw among the survivors
  const int slot = trace_pre(s);
  e = launch_k(klg::filter_select_kernel, dim3((unsigned)n_rows), dim3(klg::FILT_THREADS), 0, s, 1,
               static_cast<const int*>(cnt), static_cast<const float*>(cz), static_cast<const int*>(ci), (int)cap,
               static_cast<const float*>(lse_all), inv_temp, top_k, top_p, (uint32_t)seed, (uint32_t)(seed >> 32), tokens,
               logit, lse, overflow);
  trace_post(slot, s, KLG_KIND_SAMPLE);
  if (e != cudaSuccess) return cuda_fail(e, "launch filter_select_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_gather_rows(const void* diff, const void* ar, const int64_t* anchors, const int64_t* targets, int64_t batch,
                    int64_t n_blocks, int64_t block, int64_t ar_len, int64_t row_bytes, int64_t pad_id, void* h_s,
                    void* h_t, uint8_t* valid, void* stream) {
  if (!diff || !ar || !anchors || !targets || !h_s || !h_t || !valid) return fail(KLG_ERR_ARG, "null pointer");
  if (batch < 1 || n_blocks < 1 || block < 2 || ar_len < 1 || row_bytes < 16 ||
      batch * n_blocks * block > (1ll << 31) || batch * ar_len > (1ll << 40))
    return fail(KLG_ERR_ARG, "bad row-selection shape");
  if (row_bytes % 16 != 0) return fail(KLG_ERR_ALIGN, "row_bytes=%lld must be a multiple of 16", (long long)row_bytes);
  for (const void* p : {diff, ar, (const void*)h_s, (const void*)h_t})
    if (!aligned16(p)) return fail(KLG_ERR_ALIGN, "rows must be 16-byte aligned");
  int rc = bind_device(diff);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const long long rows = batch * n_blocks * (block - 1);
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::gather_rows_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, s, 1,
                           static_cast<const uint8_t*>(diff), static_cast<const uint8_t*>(ar),
                           reinterpret_cast<const long long*>(anchors), reinterpret_cast<const long long*>(targets),
                           (int)batch, (int)n_blocks, (int)block, (int)ar_len, (int)row_bytes, (long long)pad_id,
                           static_cast<uint8_t*>(h_s), static_cast<uint8_t*>(h_t), valid);
  trace_post(slot, s, KLG_KIND_GATHER);
  if (e != cudaSuccess) return cuda_fail(e, "launch gather_rows_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_scatter_rows_grad(const void* d_hs, int64_t batch, int64_t n_blocks, int64_t block, int64_t row_bytes,
                          void* d_diff, void* stream) {
  if (!d_hs || !d_diff) return fail(KLG_ERR_ARG, "null pointer");
  if (batch < 1 || n_blocks < 1 || block < 2 || row_bytes < 16 || batch * n_blocks * block > (1ll << 31))
    return fail(KLG_ERR_ARG, "bad row-selection shape");
  if (row_bytes % 16 != 0 || !aligned16(d_hs) || !aligned16(d_diff))
    return fail(KLG_ERR_ALIGN, "rows must be 16-byte aligned, row_bytes a multiple of 16");
  int rc = bind_device(d_hs);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const long long rows = batch * n_blocks * block;
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::scatter_rows_grad_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, s, 1,
                           static_cast<const uint8_t*>(d_hs), (int)batch, (int)n_blocks, (int)block, (int)row_bytes,
                           static_cast<uint8_t*>(d_diff));
  trace_post(slot, s, KLG_KIND_GATHER);
  if (e != cudaSuccess) return cuda_fail(e, "launch scatter_rows_grad_kernel");
  ++g_launches;
  return KLG_OK;
}

namespace {
int check_norm(const void* x, int x_f32, const float* gamma, int64_t n_rows, int64_t hidden) {
  if (!x || !gamma) return fail(KLG_ERR_ARG, "null input pointer");
  if (x_f32 != 0 && x_f32 != 1) return fail(KLG_ERR_ARG, "x_f32 must be 0 (bf16) or 1 (fp32)");
  if (n_rows < 1 || hidden < 8 || n_rows > (1ll << 30) || hidden > (1ll << 20))
    return fail(KLG_ERR_ARG, "bad shape N=%lld H=%lld", (long long)n_rows, (long long)hidden);
  if (hidden % 8 != 0) return fail(KLG_ERR_ALIGN, "hidden=%lld must be a multiple of 8", (long long)hidden);
  if (!aligned16(x) || !aligned16(gamma)) return fail(KLG_ERR_ALIGN, "x and gamma must be 16-byte aligned");
  return KLG_OK;
}
}  // namespace

int klg_rmsnorm_rows(const void* x, int x_f32, const float* gamma, int64_t n_rows, int64_t hidden, float eps, void* y,
                     float* rstd, void* stream) {
  int rc = check_norm(x, x_f32, gamma, n_rows, hidden);
  if (rc) return rc;
  if (!y || !aligned16(y)) return fail(KLG_ERR_ALIGN, "y must be non-null and 16-byte aligned");
  if (!(eps >= 0.f) || !std::isfinite(eps)) return fail(KLG_ERR_ARG, "eps must be finite and >= 0");
  if ((rc = bind_device(x))) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int slot = trace_pre(s);
  auto k = x_f32 ? klg::rmsnorm_rows_kernel<true> : klg::rmsnorm_rows_kernel<false>;
  cudaError_t e = launch_k(k, dim3(cdiv(n_rows, 8)), dim3(256), 0, s, 1, x, gamma, (int)n_rows, (int)hidden, eps,
                           static_cast<__nv_bfloat16*>(y), rstd);
  trace_post(slot, s, KLG_KIND_NORM);
  if (e != cudaSuccess) return cuda_fail(e, "launch rmsnorm_rows_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_rmsnorm_rows_bwd(const void* x, int x_f32, const float* gamma, const float* rstd, const float* dy,
                         int64_t n_rows, int64_t hidden, float* dx, void* stream) {
  int rc = check_norm(x, x_f32, gamma, n_rows, hidden);
  if (rc) return rc;
  if (!rstd || !dy || !dx) return fail(KLG_ERR_ARG, "null rstd/dy/dx");
  if (!aligned16(dy) || !aligned16(dx)) return fail(KLG_ERR_ALIGN, "dy and dx must be 16-byte aligned");
  if ((rc = bind_device(x))) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int slot = trace_pre(s);
  auto k = x_f32 ? klg::rmsnorm_rows_bwd_kernel<true> : klg::rmsnorm_rows_bwd_kernel<false>;
  cudaError_t e = launch_k(k, dim3(cdiv(n_rows, 8)), dim3(256), 0, s, 1, x, gamma, rstd, dy, (int)n_rows, (int)hidden,
                           dx);
  trace_post(slot, s, KLG_KIND_NORM);
  if (e != cudaSuccess) return cuda_fail(e, "launch rmsnorm_rows_bwd_kernel");
  ++g_launches;
  return KLG_OK;
}

// ---------------------------------------------------------------- block-diffusion attention
namespace {
struct AttnPlan {
  klg::AttnArgs a;
  int64_t ws_bytes;
};

// Largest cluster size (8, 4 or 2; else 1) whose CTAs of block_attn_kernel can all be resident
// on the current device at once (cudaOccupancyMaxActiveClusters >= 1), memoised per device;
// 8, the portable maximum, when the device cannot be queried (no device bound yet).
int attn_max_cluster() {
  static std::mutex mu;
  static std::map<int, int> memo;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 8;
  }
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(dev);
    if (it != memo.end()) return it->second;
  }
  if (set_smem(klg::block_attn_kernel, klg::ATT_SMEM) != cudaSuccess) {
    cudaGetLastError();
    return 8;
  }
  int best = 1;
  for (int c = 8; c >= 2; c >>= 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c);
    cfg.blockDim = dim3(klg::ATT_THREADS);
    cfg.dynamicSmemBytes = klg::ATT_SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = c;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, klg::block_attn_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      return 8;
    }
    if (n >= 1) {
      best = c;
      break;
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  memo[dev] = best;
  return best;
}

int attn_plan(int64_t B, int64_t H, int64_t Hkv, int64_t Ld, int64_t K, int64_t ar_len, int64_t head_dim,
              AttnPlan& P) {
  if (B < 1 || H < 1 || Hkv < 1 || Ld < 1 || K < 1 || ar_len < 1)
    return fail(KLG_ERR_ARG, "bad attention shape B=%lld H=%lld Hkv=%lld Ld=%lld K=%lld ar_len=%lld", (long long)B,
                (long long)H, (long long)Hkv, (long long)Ld, (long long)K, (long long)ar_len);
  if (head_dim != klg::ATT_D) return fail(KLG_ERR_ARG, "head_dim=%lld: only 64 is built", (long long)head_dim);
  if (K % 16 != 0 || K > 128) return fail(KLG_ERR_ARG, "block size K=%lld must be a multiple of 16 and <= 128", (long long)K);
  if (Ld % K != 0) return fail(KLG_ERR_ARG, "diffusion length %lld is not a multiple of K=%lld", (long long)Ld, (long long)K);
  if (H % Hkv != 0) return fail(KLG_ERR_ARG, "H=%lld is not a multiple of Hkv=%lld", (long long)H, (long long)Hkv);
  if (B * H * Ld > (1ll << 31) || ar_len > (1 << 24) || B * Hkv > (1 << 20))
    return fail(KLG_ERR_ARG, "attention shape too large");
  klg::AttnArgs& a = P.a;
  a = klg::AttnArgs{};
  a.B = (int)B; a.H = (int)H; a.Hkv = (int)Hkv; a.Ld = (int)Ld; a.K = (int)K; a.ar_len = (int)ar_len;
  a.ng = (int)(H / Hkv);
  a.hg = 1;
  for (int d = 1; d <= a.ng; ++d)
    if (a.ng % d == 0 && d * a.K <= 128) a.hg = d;
  a.n_hg = a.ng / a.hg;
  a.nb = (int)(Ld / K);
  a.n_units = a.B * a.Hkv * a.n_hg * a.nb;
  const int n_ar = cdiv(ar_len, klg::ATT_BN);
  // few units (decode): split the AR keys over a cluster of up to 8 CTAs (the portable
  // cluster size, or the largest that fits on the device), aiming at about two CTAs per SM
  int splits = cdiv(2 * num_sms(), a.n_units);
  splits = std::max(1, std::min(std::min(splits, n_ar), attn_max_cluster()));
  a.tps = cdiv(n_ar, splits);
  a.splits = cdiv(n_ar, a.tps);
  a.stall_split = -1;
  P.ws_bytes = 16;   // the splits combine through distributed shared memory: no global scratch
  return KLG_OK;
}
}  // namespace

int64_t klg_block_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t kv_heads, int64_t diff_len,
                                       int64_t block, int64_t ar_len, int64_t head_dim) {
  AttnPlan P;
  if (attn_plan(batch, heads, kv_heads, diff_len, block, ar_len, head_dim, P)) return -1;
  return P.ws_bytes;
}

namespace {
int block_attn_fwd(const void* q, const void* k_self, const void* v_self, const void* k_ar, const void* v_ar,
                   int64_t ar_stride, const int32_t* limits, int64_t batch, int64_t heads, int64_t kv_heads,
                   int64_t diff_len, int64_t block, int64_t ar_len, int64_t head_dim, float scale, void* out,
                   float* lse, void* workspace, int64_t workspace_bytes, void* stream, int stall_split) {
  if (!q || !k_self || !v_self || !k_ar || !v_ar || !limits || !out) return fail(KLG_ERR_ARG, "null pointer");
  AttnPlan P;
  int rc = attn_plan(batch, heads, kv_heads, diff_len, block, ar_len, head_dim, P);
  if (rc) return rc;
  if (ar_stride < ar_len) return fail(KLG_ERR_ARG, "ar_stride %lld < ar_len %lld", (long long)ar_stride, (long long)ar_len);
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(KLG_ERR_ARG, "scale must be finite and > 0");
  for (const void* p : {q, k_self, v_self, k_ar, v_ar, (const void*)out})
    if (!aligned16(p)) return fail(KLG_ERR_ALIGN, "q/k/v/out must be 16-byte aligned");
  if (!workspace || !aligned16(workspace) || workspace_bytes < P.ws_bytes)
    return fail(KLG_ERR_WORKSPACE, "attention workspace needs %lld bytes (16-byte aligned)", (long long)P.ws_bytes);
  if ((rc = bind_device(q))) return rc;
  NvtxRange nvtx_range("klg_block_attn_fwd");
  cudaStream_t s = (cudaStream_t)stream;
  klg::AttnArgs a = P.a;
  if (stall_split >= 0) {
    if (a.splits < 2 || stall_split >= a.splits)
      return fail(KLG_ERR_ARG, "stall_split %d needs a decode shape with more splits (this one has %d)", stall_split,
                  a.splits);
    a.stall_split = stall_split;
  }
  a.limits = limits;
  a.sl2 = scale * 1.4426950408889634f;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  const int D = klg::ATT_D;
  alignas(64) CUtensorMap mq, mks, mvs, mka, mva;
  if (!make_map(&mq, q, D, (uint64_t)batch * heads * diff_len, D, D, (uint32_t)block) ||
      !make_map(&mks, k_self, D, (uint64_t)batch * kv_heads * diff_len, D, D, (uint32_t)block) ||
      !make_map(&mvs, v_self, D, (uint64_t)batch * kv_heads * diff_len, D, D, (uint32_t)block) ||
      !make_map_3d(&mka, k_ar, D, ar_len, (uint64_t)batch * kv_heads, D, (uint64_t)ar_stride * D, D, klg::ATT_BN) ||
      !make_map_3d(&mva, v_ar, D, ar_len, (uint64_t)batch * kv_heads, D, (uint64_t)ar_stride * D, D, klg::ATT_BN))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  cudaError_t e = set_smem(klg::block_attn_kernel, klg::ATT_SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(block_attn_kernel)");
  int slot = trace_pre(s);
  e = launch_k(klg::block_attn_kernel, dim3(a.n_units * a.splits), dim3(klg::ATT_THREADS), klg::ATT_SMEM, s, a.splits,
               mq, mks, mvs, mka, mva, a);
  trace_post(slot, s, KLG_KIND_ATTN);
  if (e != cudaSuccess) return cuda_fail(e, "launch block_attn_kernel");
  ++g_launches;
  return KLG_OK;
}
}  // namespace

int klg_block_attn_fwd(const void* q, const void* k_self, const void* v_self, const void* k_ar, const void* v_ar,
                       int64_t ar_stride, const int32_t* limits, int64_t batch, int64_t heads, int64_t kv_heads,
                       int64_t diff_len, int64_t block, int64_t ar_len, int64_t head_dim, float scale, void* out,
                       float* lse, void* workspace, int64_t workspace_bytes, void* stream) {
  return block_attn_fwd(q, k_self, v_self, k_ar, v_ar, ar_stride, limits, batch, heads, kv_heads, diff_len, block,
                        ar_len, head_dim, scale, out, lse, workspace, workspace_bytes, stream, -1);
}

int klg_selftest_attn_split_stall(const void* q, const void* k_self, const void* v_self, const void* k_ar,
                                  const void* v_ar, int64_t ar_stride, const int32_t* limits, int64_t batch,
                                  int64_t heads, int64_t kv_heads, int64_t diff_len, int64_t block, int64_t ar_len,
                                  int64_t head_dim, float scale, void* out, float* lse, void* workspace,
                                  int64_t workspace_bytes, int stall_split, void* stream) {
  if (stall_split < 0) return fail(KLG_ERR_ARG, "stall_split must be >= 0");
  return block_attn_fwd(q, k_self, v_self, k_ar, v_ar, ar_stride, limits, batch, heads, kv_heads, diff_len, block,
                        ar_len, head_dim, scale, out, lse, workspace, workspace_bytes, stream, stall_split);
}

int klg_block_attn_splits(int64_t batch, int64_t heads, int64_t kv_heads, int64_t diff_len, int64_t block,
                          int64_t ar_len, int64_t head_dim) {
  AttnPlan P;
  if (attn_plan(batch, heads, kv_heads, diff_len, block, ar_len, head_dim, P)) return -1;
  return P.a.splits;
}

int klg_block_attn_bwd(const void* q, const void* k_self, const void* v_self, const void* k_ar, const void* v_ar,
                       int64_t ar_stride, const int32_t* limits, const void* out, const float* lse, const void* d_out,
                       int64_t batch, int64_t heads, int64_t kv_heads, int64_t diff_len, int64_t block, int64_t ar_len,
                       int64_t head_dim, float scale, float* d_q, float* d_k_self, float* d_v_self, void* stream) {
  if (!q || !k_self || !v_self || !k_ar || !v_ar || !limits || !out || !lse || !d_out || !d_q || !d_k_self || !d_v_self)
    return fail(KLG_ERR_ARG, "null pointer");
  AttnPlan P;
  int rc = attn_plan(batch, heads, kv_heads, diff_len, block, ar_len, head_dim, P);
  if (rc) return rc;
  if (ar_stride < ar_len) return fail(KLG_ERR_ARG, "ar_stride %lld < ar_len %lld", (long long)ar_stride, (long long)ar_len);
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(KLG_ERR_ARG, "scale must be finite and > 0");
  for (const void* p : {q, k_self, v_self, k_ar, v_ar, out, d_out, (const void*)d_q, (const void*)d_k_self,
                        (const void*)d_v_self})
    if (!aligned16(p)) return fail(KLG_ERR_ALIGN, "q/k/v/out/gradients must be 16-byte aligned");
  if ((rc = bind_device(q))) return rc;
  NvtxRange nvtx_range("klg_block_attn_bwd");
  cudaStream_t s = (cudaStream_t)stream;
  const klg::AttnArgs& f = P.a;
  klg::AttnBwdArgs a{};
  a.limits = limits;
  a.out = static_cast<const __nv_bfloat16*>(out);
  a.dout = static_cast<const __nv_bfloat16*>(d_out);
  a.lse = lse;
  a.dq = d_q;
  a.dk = d_k_self;
  a.dv = d_v_self;
  a.B = f.B; a.H = f.H; a.Hkv = f.Hkv; a.Ld = f.Ld; a.K = f.K; a.ar_len = f.ar_len;
  a.ng = f.ng; a.hg = f.hg; a.n_hg = f.n_hg; a.nb = f.nb; a.n_units = f.n_units;
  a.scale = scale;
  a.sl2 = scale * 1.4426950408889634f;
  a.accumulate_kv = f.n_hg > 1;
  if (a.accumulate_kv) {   // several head groups add into the same self keys' dk / dv
    const long long n4 = (long long)batch * kv_heads * diff_len * head_dim / 4;
    for (float* buf : {d_k_self, d_v_self}) {
      const int blocks = (int)std::min<long long>(cdiv(n4, 256), 4ll * num_sms());
      cudaError_t ze = launch_k(klg::zero_f32x4_kernel, dim3(blocks), dim3(256), 0, s, 1, reinterpret_cast<float4*>(buf), n4);
      if (ze != cudaSuccess) return cuda_fail(ze, "launch zero_f32x4_kernel");
      ++g_launches;
    }
  }
  const int D = klg::ATT_D;
  alignas(64) CUtensorMap mq, mdo, mks, mvs, mka, mva;
  if (!make_map(&mq, q, D, (uint64_t)batch * heads * diff_len, D, D, (uint32_t)block) ||
      !make_map(&mdo, d_out, D, (uint64_t)batch * heads * diff_len, D, D, (uint32_t)block) ||
      !make_map(&mks, k_self, D, (uint64_t)batch * kv_heads * diff_len, D, D, (uint32_t)block) ||
      !make_map(&mvs, v_self, D, (uint64_t)batch * kv_heads * diff_len, D, D, (uint32_t)block) ||
      !make_map_3d(&mka, k_ar, D, ar_len, (uint64_t)batch * kv_heads, D, (uint64_t)ar_stride * D, D, klg::ATT_BN) ||
      !make_map_3d(&mva, v_ar, D, ar_len, (uint64_t)batch * kv_heads, D, (uint64_t)ar_stride * D, D, klg::ATT_BN))
    return fail(KLG_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  cudaError_t e = set_smem(klg::block_attn_bwd_kernel, klg::ATB_SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(block_attn_bwd_kernel)");
  const int slot = trace_pre(s);
  e = launch_k(klg::block_attn_bwd_kernel, dim3(a.n_units), dim3(klg::ATB_THREADS), klg::ATB_SMEM, s, 1, mq, mdo, mks,
               mvs, mka, mva, a);
  trace_post(slot, s, KLG_KIND_ATTN);
  if (e != cudaSuccess) return cuda_fail(e, "launch block_attn_bwd_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_token_logit(const void* h, const void* w, const int32_t* tokens, int64_t n_rows, int64_t hidden, int64_t vocab,
                    float* z, void* stream) {
  if (!h || !w || !tokens || !z) return fail(KLG_ERR_ARG, "null pointer");
  if (n_rows < 1 || hidden < 8 || vocab < 1 || n_rows > (1ll << 30) || hidden > (1ll << 20) || vocab > (1ll << 30))
    return fail(KLG_ERR_ARG, "bad shape N=%lld H=%lld V=%lld", (long long)n_rows, (long long)hidden, (long long)vocab);
  if (hidden % 8 != 0 || !aligned16(h) || !aligned16(w))
    return fail(KLG_ERR_ALIGN, "hidden must be a multiple of 8 and rows 16-byte aligned");
  int rc = bind_device(h);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int slot = trace_pre(s);
  cudaError_t e = launch_k(klg::token_logit_kernel, dim3(cdiv(n_rows, 8)), dim3(256), 0, s, 1,
                           static_cast<const __nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(w), tokens,
                           (int)n_rows, (int)hidden, (int)vocab, z);
  trace_post(slot, s, KLG_KIND_SAMPLE);
  if (e != cudaSuccess) return cuda_fail(e, "launch token_logit_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_cast_f32_bf16(const float* in, void* out, int64_t n, void* stream) {
  if (!in || !out || n < 0) return fail(KLG_ERR_ARG, "bad arguments to klg_cast_f32_bf16");
  if (n == 0) return KLG_OK;
  if (int rc = bind_device(in)) return rc;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  const int slot = trace_pre((cudaStream_t)stream);
  cudaError_t e = launch_k(klg::cast_f32_bf16_kernel, dim3((int)blocks), dim3(256), 0, (cudaStream_t)stream, 1, in,
                           static_cast<__nv_bfloat16*>(out), n);
  trace_post(slot, (cudaStream_t)stream, KLG_KIND_CAST);
  if (e != cudaSuccess) return cuda_fail(e, "launch cast_f32_bf16_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_scale_cast(const float* in, const float* g, int64_t n, void* out, int out_bf16, void* stream) {
  if (!in || !out || n < 0) return fail(KLG_ERR_ARG, "bad arguments to klg_scale_cast");
  if (!aligned16(in) || !aligned16(out)) return fail(KLG_ERR_ALIGN, "klg_scale_cast: in and out must be 16-byte aligned");
  if (n == 0) return KLG_OK;
  if (int rc = bind_device(in)) return rc;
  long long blocks = (n / 4 + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 4ll * num_sms()) blocks = 4ll * num_sms();
  const int slot = trace_pre((cudaStream_t)stream);
  cudaError_t e = launch_k(klg::scale_cast_kernel, dim3((int)blocks), dim3(256), 0, (cudaStream_t)stream, 1, in, g,
                           (long long)n, out, out_bf16);
  trace_post(slot, (cudaStream_t)stream, KLG_KIND_CAST);
  if (e != cudaSuccess) return cuda_fail(e, "launch scale_cast_kernel");
  ++g_launches;
  return KLG_OK;
}

int klg_trace_begin(int capacity) {
  if (capacity < 1 || capacity > (1 << 20)) return fail(KLG_ERR_ARG, "trace capacity out of range");
  std::lock_guard<std::mutex> lk(g_trace.mu);
  while ((int)g_trace.ev.size() < 2 * capacity) {
    cudaEvent_t e;
    cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) return cuda_fail(err, "cudaEventCreate");
    g_trace.ev.push_back(e);
  }
  g_trace.kind.assign(capacity, 0);
  g_trace.cap = capacity;
  g_trace.used = 0;
  g_trace.on = true;
  return KLG_OK;
}

int klg_trace_end(int* kinds, float* ms, int capacity, int* n) {
  std::lock_guard<std::mutex> lk(g_trace.mu);
  g_trace.on = false;
  const int used = g_trace.used;
  if (n) *n = used;
  for (int i = 0; i < used && i < capacity; ++i) {
    cudaError_t err = cudaEventSynchronize(g_trace.ev[2 * i + 1]);
    if (err != cudaSuccess) return cuda_fail(err, "cudaEventSynchronize");
    float t = 0.f;
    err = cudaEventElapsedTime(&t, g_trace.ev[2 * i], g_trace.ev[2 * i + 1]);
    if (err != cudaSuccess) return cuda_fail(err, "cudaEventElapsedTime");
    if (kinds) kinds[i] = g_trace.kind[i];
    if (ms) ms[i] = t;
  }
  g_trace.used = 0;
  return used > capacity ? fail(KLG_ERR_ARG, "trace holds %d launches, buffer %d", used, capacity) : KLG_OK;
}

}  // extern "C"

// ============================================================ allocation-free forward
//
// klg_fwd_noalloc: the forward of klg_fwd for callers that cannot allocate device
// memory -- for example a host runtime whose device memory is entirely reserved
// up front by its own allocator (so there is nowhere to put a workspace), or a
// call site on a latency-critical loop where cudaMalloc's implicit device-wide
// synchronisation is not acceptable.  Instead of a caller-provided workspace the
// pass-1 partial records and the merged row statistics live in the file-scope
// array below, which every GPU that loads this library keeps for the life of the
// process (KLG_NOALLOC_SCRATCH_FLOATS floats = 16 MiB).
//
// Host code never uses `klg_noalloc_scratch` as an address: on the host that name
// only stands for the device variable.  The device address is looked up once per
// device with cudaGetSymbolAddress (with that device current) on the first call
// made on that device, so make that first call before any stream capture.  All
// calls share the one array and it keeps the last call's contents; nothing in it
// needs to start at zero (every call overwrites what it reads).  Calls whose work
// overlaps on the GPU (different streams, or several host threads) race on it.

#define KLG_NOALLOC_SCRATCH_FLOATS (4ll << 20)

static __device__ __align__(256) float klg_noalloc_scratch[KLG_NOALLOC_SCRATCH_FLOATS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up on first use).
int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(KLG_ERR_ARG, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, klg_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(klg_noalloc_scratch)");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return KLG_OK;
}

}  // namespace

extern "C" {

long long klg_fwd_noalloc_max_floats(void) { return KLG_NOALLOC_SCRATCH_FLOATS; }

int klg_fwd_noalloc(const void* hs, const void* ht, const void* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
                    int64_t vocab, float inv_temp, int count_given, float* count, float* loss, float* lse,
                    float* row_kl, void* stream) {
  int rc = check_problem(hs, ht, w, n_rows, hidden, vocab, inv_temp);
  if (rc) return rc;
  if (!mask || !count || !loss || !lse) return fail(KLG_ERR_ARG, "null output pointer");
  if ((rc = bind_device(hs))) return rc;   // the partial-record count depends on hs's device
  int n_part = 0;
  if ((rc = klg_num_partials(n_rows, vocab, &n_part))) return rc;
  const long long need = (long long)(n_part + 1) * 5 * n_rows;
  if (need > KLG_NOALLOC_SCRATCH_FLOATS)
    return fail(KLG_ERR_WORKSPACE,
                "klg_fwd_noalloc: %lld rows x %lld vocab needs %lld scratch floats, above its fixed %lld "
                "(use klg_fwd with a workspace)",
                (long long)n_rows, (long long)vocab, need, (long long)KLG_NOALLOC_SCRATCH_FLOATS);
  float* parts = nullptr;
  if ((rc = noalloc_scratch(&parts))) return rc;
  float* stats = parts + (size_t)n_part * 5 * n_rows;
  if (!count_given && (rc = klg_count_valid(mask, n_rows, count, stream))) return rc;
  if ((rc = klg_fwd_stats(hs, ht, w, n_rows, hidden, vocab, inv_temp, parts, n_part, stream))) return rc;
  if ((rc = klg_merge_stats(parts, n_part, n_rows, stats, stream))) return rc;
  return klg_finalize(stats, mask, n_rows, count, loss, lse, row_kl, stream);
}

}  // extern "C"
