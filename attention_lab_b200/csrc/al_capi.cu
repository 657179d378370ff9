// C ABI of the sparse-decode library: validation, launch-shape choice and template dispatch.
// Declarations and contracts: include/attention_lab_b200.h.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "al_context.cuh"
#include "al_index.cuh"
#include "al_prefill.cuh"
#include "../../include/attention_lab_b200.h"

namespace al {
__device__ unsigned g_al_error;   // kernel error bits (see kErr*)
}

using namespace al;

namespace {

thread_local char g_msg[1024] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(AL_ECUDA, "%s: %s", where, cudaGetErrorString(e));
}

constexpr int kMaxRanks = 64;   // ranks of one exchange (the flag array of a channel holds one word each)

struct DeviceInfo {
  int sms = 0;
  int max_smem_optin = 0;
  unsigned* err = nullptr;
};

std::mutex g_mu;
DeviceInfo g_dev[64];
std::unordered_map<unsigned long long, int> g_smem_set;   // (kernel, device) -> dynamic smem bytes allowed

int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(AL_ECUDA, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.err) {
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    if ((e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(max shared memory)");
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_al_error)) != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    d.err = static_cast<unsigned*>(p);
  }
  *out = &d;
  return AL_OK;
}

template <typename K>
int prepare_kernel(K kernel, size_t smem, int cs) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long key = (reinterpret_cast<unsigned long long>(reinterpret_cast<const void*>(kernel)) << 6) ^
                                 (unsigned long long)dev;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_smem_set.find(key);
  if (it == g_smem_set.end() || it->second < (int)smem) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic shared memory)");
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(non-portable cluster)");
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(shared memory carve-out)");
    g_smem_set[key] = (int)smem;
  }
  (void)cs;
  return AL_OK;
}

std::unordered_map<unsigned long long, int> g_cluster_ok;   // (kernel, cs, smem, device) -> schedulable

template <typename K, typename... P>
int launch(K kernel, dim3 grid, int cs, size_t smem, void* stream, const P&... p) {
  int rc = prepare_kernel(kernel, smem, cs);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cs > 1) {
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long key = (reinterpret_cast<unsigned long long>(reinterpret_cast<const void*>(kernel)) << 16) ^
                                   ((unsigned long long)cs << 40) ^ ((unsigned long long)smem << 8) ^ (unsigned long long)dev;
    int ok = -1;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_cluster_ok.find(key);
      if (it != g_cluster_ok.end()) ok = it->second;
    }
    if (ok < 0) {
      int n = 0;
      cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
      ok = n > 0 ? 1 : 0;
      std::lock_guard<std::mutex> lk(g_mu);
      g_cluster_ok[key] = ok;
    }
    if (!ok) return fail(AL_EUNSUPPORTED, "a cluster of %d CTAs with %zu bytes of shared memory cannot be scheduled", cs, smem);
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p...);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx");
  return AL_OK;
}

int plain_launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return AL_OK;
}

bool dtype_ok(int t) { return t == AL_F32 || t == AL_BF16; }
int esize(int t) { return t == AL_F32 ? 4 : 2; }
int pad_heads(int h) { return h <= 1 ? 1 : (h <= 2 ? 2 : 4); }
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Static shared memory of the fused kernel (upper bound used for the dynamic budget).
constexpr int kFusedStaticBytes = 8 * 1024;
constexpr int kAttendStaticBytes = 4 * 1024;

// Attend pipeline depth (32 KB stages). Three stages keep a CTA of the fused or the attend kernel within half of an
// SM's shared memory, so two 256-thread CTAs share each SM (measured: six 16 KB stages of 64-row tiles ran slower,
// the engine is bound by its per-tile work rather than by the bytes in flight).
constexpr int kStages = 3;
constexpr int kFusedStages = 3;
// Dynamic shared memory of one CTA when two share an SM: half of the SM's 228 KB, less the 1 KB the runtime reserves
// per CTA and a 4 KB allowance for the kernels' static shared memory.
constexpr long long kHalfSmBudget = 228 * 1024 / 2 - 1024 - 4096;

int engine_smem(int kv_dtype, int hp, int stages = kStages) {
  switch (kv_dtype * 8 + hp) {
    case AL_F32 * 8 + 1: return AttendCfg<float, 1>::smem(stages);
    case AL_F32 * 8 + 2: return AttendCfg<float, 2>::smem(stages);
    case AL_F32 * 8 + 4: return AttendCfg<float, 4>::smem(stages);
    case AL_BF16 * 8 + 1: return AttendCfg<__nv_bfloat16, 1>::smem(stages);
    case AL_BF16 * 8 + 2: return AttendCfg<__nv_bfloat16, 2>::smem(stages);
    default: return AttendCfg<__nv_bfloat16, 4>::smem(stages);
  }
}

// Automatic cluster size: more CTAs per segment while the grid does not cover the SMs, up to kAutoCluster (measured
// at batch 1: clusters of 16 spend more on cluster synchronisation than the extra CTAs return; C4 113 -> 76 us,
// C2 1.04 -> 0.97 ms per step with 8), and few enough keys per CTA to fit shared memory.
constexpr int kAutoCluster = 8;
int auto_cluster(int segs, int M, int sms, int max_keys) {
  int cs = 1;
  while (cs < kMaxCluster && (long long)M > (long long)cs * max_keys) cs <<= 1;
  while (cs < kAutoCluster && segs * cs < sms && M / (cs * 2) >= 256) cs <<= 1;
  return cs;
}

template <typename KV_T, typename IDX_T>
int dispatch_fused_h(const DecodeParams& p, const CUtensorMap& zmap, int hp, dim3 grid, int cs, size_t smem,
                     void* stream) {
  switch (hp) {
    case 1: return launch(sparse_step_kernel<KV_T, IDX_T, 1>, grid, cs, smem, stream, p, zmap);
    case 2: return launch(sparse_step_kernel<KV_T, IDX_T, 2>, grid, cs, smem, stream, p, zmap);
    default: return launch(sparse_step_kernel<KV_T, IDX_T, 4>, grid, cs, smem, stream, p, zmap);
  }
}

int dispatch_fused(const DecodeParams& p, const CUtensorMap& zmap, int kv_dtype, int idx_dtype, int hp, dim3 grid,
                   int cs, size_t smem, void* stream) {
  if (kv_dtype == AL_BF16 && idx_dtype == AL_F32)
    return dispatch_fused_h<__nv_bfloat16, float>(p, zmap, hp, grid, cs, smem, stream);
  if (kv_dtype == AL_BF16 && idx_dtype == AL_BF16)
    return dispatch_fused_h<__nv_bfloat16, __nv_bfloat16>(p, zmap, hp, grid, cs, smem, stream);
  if (kv_dtype == AL_F32 && idx_dtype == AL_F32) return dispatch_fused_h<float, float>(p, zmap, hp, grid, cs, smem, stream);
  return dispatch_fused_h<float, __nv_bfloat16>(p, zmap, hp, grid, cs, smem, stream);
}

// Tensor map of an index table zT [B,G,r,C] viewed as [B*G*r rows, C columns] with boxes of 32 rows x 512 bytes
// (the resident-key scan's tiles). The driver's encoder is reached through the runtime (no libcuda link); maps are
// cached by (address, shape, dtype). Returns false when the encoder is unavailable or refuses the layout.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::unordered_map<unsigned long long, CUtensorMap> g_zmaps;

EncodeTiledFn tensor_map_encoder() {   // called with g_mu held
  static EncodeTiledFn enc = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      enc = reinterpret_cast<EncodeTiledFn>(fn);
  }
  return enc;
}

bool zt_tensor_map(const void* zT, int idx_dtype, long long rows, int C, CUtensorMap* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  const EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return false;
  const unsigned long long key = reinterpret_cast<unsigned long long>(zT) ^ ((unsigned long long)C << 1) ^
                                 ((unsigned long long)rows << 29) ^ ((unsigned long long)idx_dtype << 62);
  auto it = g_zmaps.find(key);
  if (it != g_zmaps.end()) { *out = it->second; return true; }
  const int es = esize(idx_dtype);
  cuuint64_t dims[2] = {(cuuint64_t)C, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)C * (cuuint64_t)es};
  cuuint32_t box[2] = {(cuuint32_t)(512 / es), 32u};
  cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  const CUresult r = enc(&m, idx_dtype == AL_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                         const_cast<void*>(zT), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (g_zmaps.size() > 4096) g_zmaps.clear();
  g_zmaps[key] = m;
  *out = m;
  return true;
}

// Tensor map of the prefill scorer's zT [H, 32, C] (bf16, element strides z_sh, z_ld): boxes of 64 columns x 32 rows
// x 1 head with the 128-byte swizzle, the N-major operand layout of the tensor-core MMA. Cached like zt_tensor_map.
std::unordered_map<unsigned long long, CUtensorMap> g_pfmaps;

bool pf_tensor_map(const void* zT, int H, int C, long long z_sh, long long z_ld, CUtensorMap* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  const EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return false;
  const unsigned long long key = reinterpret_cast<unsigned long long>(zT) ^ ((unsigned long long)C << 1) ^
                                 ((unsigned long long)H << 20) ^ ((unsigned long long)z_sh << 30) ^
                                 ((unsigned long long)z_ld << 47);
  auto it = g_pfmaps.find(key);
  if (it != g_pfmaps.end()) { *out = it->second; return true; }
  cuuint64_t dims[3] = {(cuuint64_t)C, 32u, (cuuint64_t)H};
  cuuint64_t strides[2] = {(cuuint64_t)z_ld * 2u, (cuuint64_t)z_sh * 2u};
  cuuint32_t box[3] = {64u, 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMap m;
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(zT), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (g_pfmaps.size() > 4096) g_pfmaps.clear();
  g_pfmaps[key] = m;
  *out = m;
  return true;
}

int dispatch_attend(const AttendParams& p, int kv_dtype, int hp, dim3 grid, int cs, size_t smem, void* stream) {
  if (kv_dtype == AL_BF16) {
    switch (hp) {
      case 1: return launch(attend_kernel<__nv_bfloat16, 1>, grid, cs, smem, stream, p);
      case 2: return launch(attend_kernel<__nv_bfloat16, 2>, grid, cs, smem, stream, p);
      default: return launch(attend_kernel<__nv_bfloat16, 4>, grid, cs, smem, stream, p);
    }
  }
  switch (hp) {
    case 1: return launch(attend_kernel<float, 1>, grid, cs, smem, stream, p);
    case 2: return launch(attend_kernel<float, 2>, grid, cs, smem, stream, p);
    default: return launch(attend_kernel<float, 4>, grid, cs, smem, stream, p);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Shared validation + launch of the fused kernel (decode step or select-only).
int run_fused(DecodeParams p, int kv_dtype, int idx_dtype, int d, int cluster, void* stream, bool attend) {
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  if (!dtype_ok(idx_dtype) || (attend && !dtype_ok(kv_dtype))) return fail(AL_EINVAL, "unknown dtype code");
  if (p.B <= 0 || p.G <= 0 || p.C <= 0) return fail(AL_EINVAL, "B, G and C must be positive");
  if (p.B * (long long)p.G > 65535) return fail(AL_EUNSUPPORTED, "B*G = %lld exceeds 65535", p.B * (long long)p.G);
  if (d != kHeadDim) return fail(AL_EUNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, d);
  if (p.r < 1 || p.r > kMaxR) return fail(AL_EUNSUPPORTED, "index width r must be in [1, %d], got %d", kMaxR, p.r);
  if (attend && (p.h < 1 || p.h > 4)) return fail(AL_EUNSUPPORTED, "heads per group must be in [1, 4], got %d", p.h);
  if (!(0 <= p.lo && p.lo <= p.hi && p.hi <= p.C))
    return fail(AL_EINVAL, "need 0 <= lo <= hi <= C, got lo=%d hi=%d C=%d", p.lo, p.hi, p.C);
  p.M = p.hi - p.lo;
  if (p.k < 0 || p.k > p.M) return fail(AL_EINVAL, "k=%d must lie in [0, hi-lo=%d]", p.k, p.M);
  if (p.F < 0 || p.S != p.F + p.k)
    return fail(AL_EINVAL, "selected_count=%d must equal fixed_count=%d + k=%d", p.S, p.F, p.k);
  if (p.S < 1) return fail(AL_EINVAL, "at least one row must be selected");
  if (p.k_new && (p.write_col < 0 || p.write_col >= p.C))
    return fail(AL_EINVAL, "write_col=%d must lie in [0, C=%d)", p.write_col, p.C);
  if (p.k_new && p.lo <= p.write_col && p.write_col < p.hi)
    return fail(AL_EINVAL, "write_col=%d must lie outside the scanned range [%d, %d)", p.write_col, p.lo, p.hi);
  const long long total = (long long)p.B * p.G * p.C;
  if (total >= 0xffffffffLL) return fail(AL_EUNSUPPORTED, "B*G*C = %lld rows exceeds 2^32-1", total);
  p.total_rows = total;
  if (!p.zT || !p.off_lo || (p.F > 0 && !p.fixed_rows)) return fail(AL_EINVAL, "null zT, off_lo or fixed_rows");
  if (attend && (!p.q || !p.k_cache || !p.v_cache || (!p.out && !p.part)))
    return fail(AL_EINVAL, "null q, cache or output pointer");
  if (attend && (!aligned16(p.k_cache) || !aligned16(p.v_cache)))
    return fail(AL_EUNSUPPORTED, "k_cache and v_cache must start on a 16-byte boundary");
  if (!p.u_in && p.k > 0 && p.k < p.M && (!p.q_pre || !p.wq_t)) return fail(AL_EINVAL, "null q_pre or wq_t");
  if (p.k_new && !p.wk) return fail(AL_EINVAL, "k_pre_new given without wk");

  p.select_mode = p.k == 0 ? 0 : (p.k == p.M ? 2 : 1);
  p.scan = (p.select_mode == 1 || p.scores_out || (p.keys_out && p.select_mode == 2)) ? 1 : 0;
  if (p.keys_out && (p.kst < p.k || p.key_pos < 0 || p.key_pos + (long long)p.C > 0xffffffffLL))
    return fail(AL_EINVAL, "key_stride=%d must be >= k=%d and key positions must fit 32 bits", p.kst, p.k);
  if (p.scan && !p.u_in && (!p.q_pre || !p.wq_t)) return fail(AL_EINVAL, "null q_pre or wq_t");
  const int ez = esize(idx_dtype);
  p.zvec = ((long long)p.C * ez % 16 == 0) && aligned16(p.zT) ? 1 : 0;
  p.uvec = (p.r == kMaxR && p.wq_t && aligned16(p.wq_t)) ? 1 : 0;

  const int hp = attend ? pad_heads(p.h) : 1;
  const int budget = di->max_smem_optin - kFusedStaticBytes;
  // Resident-key scan (select_mode 1, r = 32, 16-byte aligned index rows, a tensor map): the index tiles stream
  // through a ring of 16 KB stages placed after the histogram (and the cluster slice), inside the attend engine's
  // footprint; every key goes to TMEM, so there is no candidate list. After the scan the bitmaps (and the per-column
  // keys of keys_out) reuse the ring. Otherwise: [histogram | cluster slice | bitmaps | candidate list].
  CUtensorMap zmap;
  std::memset(&zmap, 0, sizeof(zmap));
  const bool tk_ok = p.select_mode == 1 && p.scan && p.r == kMaxR && p.zvec &&
                     zt_tensor_map(p.zT, idx_dtype, (long long)p.B * p.G * p.r, p.C, &zmap);
  // Shared memory per CTA: the selection region aliased with the attend engine, then the attend row list. The list
  // path's candidate list takes whatever the engine leaves, and at least room for a typical filtered list (the first
  // scan round, plus about ln(columns / round) * k later keys). The cluster size is the automatic (or requested) one,
  // grown while a CTA's share does not fit.
  int cs = cluster > 0 ? cluster : auto_cluster(p.B * p.G, p.M, di->sms, 1 << 30);
  if (cs < 1 || cs > kMaxCluster) return fail(AL_EINVAL, "cluster must be in [1, %d], got %d", kMaxCluster, cs);
  const int round_cols = kThreads * (p.zvec ? 16 / ez : 1);
  size_t smem = 0;
  for (;; cs <<= 1) {
    p.cpc = (int)round_up((size_t)((p.M + cs - 1) / cs), 8);
    if (p.cpc == 0) p.cpc = 8;
    size_t sel_fixed = 0;
    int cap_min = 0;
    p.tkeys = tk_ok && p.cpc + 32 <= kTkeyMaxCols ? 1 : 0;
    if (p.select_mode == 1) {
      if (p.cpc > 65535) { if (cluster > 0 || cs >= kMaxCluster) return fail(AL_EUNSUPPORTED, "more than 65535 candidates per CTA (cluster %d)", cs); continue; }
      p.nwp = (p.cpc + 30) / 32 + 1;
      const int slice = cs > 1 ? (int)round_up((size_t)(4096 / cs) * 4, 16) : 0;
      if (p.tkeys) {
        // during the scan: [packed histogram 8 KB | ring]; after it: [histogram | cluster slice | bitmaps]
        p.ring_off = 2048 * 4;
        p.bm_off = 4096 * 4 + slice;
        sel_fixed = (size_t)p.bm_off + round_up((size_t)p.nwp * 8, 16);
      } else {
        p.bm_off = 4096 * 4 + slice;
        p.list_off = p.bm_off + (int)round_up((size_t)p.nwp * 8, 16);
        sel_fixed = (size_t)p.list_off;
        cap_min = std::min(p.cpc, round_cols + 6 * p.k + 1024);
      }
    }
    const int rows_cap = (p.F + cs - 1) / cs + (p.k < p.cpc ? p.k : p.cpc) + 8;
    // the deepest pipeline that leaves room for two CTAs per SM, else the deepest that fits at all
    bool fits = false;
    for (int pass = 0; pass < 2 && !fits; ++pass)
    for (int st = kFusedStages; st >= 3 && !fits; --st) {
      const size_t eng = attend ? (size_t)engine_smem(kv_dtype, hp, st) : 0;
      p.cap = 0;
      size_t select_bytes = sel_fixed;
      if (p.select_mode == 1 && !p.tkeys) {
        const size_t room = eng > sel_fixed ? (eng - sel_fixed) / 8 : 0;
        p.cap = (int)std::min<size_t>((size_t)p.cpc, std::max<size_t>(room, (size_t)cap_min));
        select_bytes += (size_t)p.cap * 8;
      }
      if (p.keys_out) {                     // per-column keys of the chosen candidates
        p.skey_off = (int)round_up(select_bytes, 16);
        select_bytes = (size_t)p.skey_off + (size_t)(p.cpc + 64) * 4;
      }
      size_t region = select_bytes > eng ? select_bytes : eng;
      if (p.tkeys) {
        // an even number of ring stages (each half of the CTA owns every other one): as many as the region holds,
        // up to kMaxRing, and kMaxRing when nothing else sets the size; the launch also keeps above a third of the
        // SM's shared memory so at most two CTAs share an SM (each holds half of its TMEM columns)
        p.nring = (int)std::min<size_t>(kMaxRing, region > (size_t)p.ring_off ? (region - p.ring_off) / kTileBytes : 0);
        if (!attend) p.nring = kMaxRing;
        p.nring &= ~1;
        if (p.nring < 2) p.nring = 2;
        region = std::max(region, (size_t)p.ring_off + (size_t)p.nring * kTileBytes);
        region = std::max(region, (size_t)80 * 1024);
        // after the scan, the candidate list of the one-CTA select (keys of the pivot bin and above) takes the rest
        p.list_off = (int)round_up(select_bytes, 16);
        p.cap = region > (size_t)p.list_off ? (int)((region - (size_t)p.list_off) / 8) : 0;
      }
      p.union_bytes = (int)round_up(region, 128);
      smem = (size_t)p.union_bytes + (size_t)rows_cap * 4;
      p.nstage = st;
      fits = (long long)smem <= (pass == 0 ? kHalfSmBudget : budget);
    }
    if (fits) break;
    if (cluster > 0 || cs >= kMaxCluster)
      return fail(AL_EUNSUPPORTED, "candidate range too large for cluster %d: %zu bytes of shared memory per CTA", cs, smem);
  }
  p.err = di->err;
  dim3 grid((unsigned)cs, (unsigned)(p.B * p.G), 1);
  if (!attend) { p.out = nullptr; p.part = nullptr; }
  return dispatch_fused(p, zmap, attend ? kv_dtype : AL_BF16, idx_dtype, hp, grid, cs, smem, stream);
}

}  // namespace

extern "C" {

const char* al_last_error(void) { return g_msg; }

int al_version(void) { return 1; }

int al_device_status(unsigned* error_bits) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned v = 0, zero = 0;
  if ((e = cudaMemcpyFromSymbol(&v, g_al_error, sizeof(v))) != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol");
  if ((e = cudaMemcpyToSymbol(g_al_error, &zero, sizeof(zero))) != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol");
  if (error_bits) *error_bits = v;
  return AL_OK;
}

int al_sparse_decode_step(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                          const void* q_pre, int64_t qp_sb, int64_t qp_sg, int64_t qp_sh,
                          const void* k_cache, const void* v_cache, int kv_dtype,
                          void* zT, const void* wq_t, const void* wk, int idx_dtype,
                          const void* k_pre_new, int64_t kn_sb, int64_t kn_sg,
                          const int64_t* fixed_rows, const int64_t* off_lo,
                          int B, int G, int h, int d, int r, int C,
                          int lo, int hi, int k, int selected_count, int fixed_count, int write_col,
                          float scale, int canonical_order,
                          void* out, int64_t* rows_out, float* scores_out, int cluster, void* stream) {
  DecodeParams p = {};
  p.B = B; p.G = G; p.h = h; p.r = r; p.C = C;
  p.lo = lo; p.hi = hi; p.k = k; p.S = selected_count; p.F = fixed_count; p.write_col = write_col;
  p.canonical = canonical_order ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = q_main; p.q_sb = q_sb; p.q_sg = q_sg; p.q_sh = q_sh;
  p.q_pre = q_pre; p.qp_sb = qp_sb; p.qp_sg = qp_sg; p.qp_sh = qp_sh;
  p.wq_t = wq_t; p.wk = wk;
  p.k_new = k_pre_new; p.kn_sb = kn_sb; p.kn_sg = kn_sg;
  p.zT = zT; p.k_cache = k_cache; p.v_cache = v_cache;
  p.fixed_rows = reinterpret_cast<const long long*>(fixed_rows);
  p.off_lo = reinterpret_cast<const long long*>(off_lo);
  p.out = out; p.rows_out = reinterpret_cast<long long*>(rows_out); p.scores_out = scores_out;
  return run_fused(p, kv_dtype, idx_dtype, d, cluster, stream, true);
}

int al_select_rows(const void* u, int64_t u_sb, int64_t u_sg, const void* zT, int idx_dtype,
                   const int64_t* fixed_rows, const int64_t* off_lo,
                   int B, int G, int r, int C, int lo, int hi, int k, int selected_count, int fixed_count,
                   int canonical_order, int64_t* rows_out, float* scores_out, int cluster, void* stream) {
  if (!rows_out) return fail(AL_EINVAL, "rows_out is required");
  if (!u) return fail(AL_EINVAL, "null u");
  if (u_sb != (int64_t)G * r || u_sg != r) return fail(AL_EINVAL, "u must be a contiguous [B,G,1,r] tensor");
  DecodeParams p = {};
  p.B = B; p.G = G; p.h = 1; p.r = r; p.C = C;
  p.lo = lo; p.hi = hi; p.k = k; p.S = selected_count; p.F = fixed_count; p.write_col = -1;
  p.canonical = canonical_order ? 1 : 0;
  p.u_in = u;
  p.zT = const_cast<void*>(zT);
  p.fixed_rows = reinterpret_cast<const long long*>(fixed_rows);
  p.off_lo = reinterpret_cast<const long long*>(off_lo);
  p.rows_out = reinterpret_cast<long long*>(rows_out); p.scores_out = scores_out;
  return run_fused(p, AL_BF16, idx_dtype, kHeadDim, cluster, stream, false);
}

static int run_attend(AttendParams p, int kv_dtype, int d, int n_all, int cluster, void* stream) {
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  if (!dtype_ok(kv_dtype)) return fail(AL_EINVAL, "unknown dtype code");
  if (p.B <= 0 || p.G <= 0 || p.C <= 0) return fail(AL_EINVAL, "B, G and C must be positive");
  if (p.B * (long long)p.G > 65535) return fail(AL_EUNSUPPORTED, "B*G exceeds 65535");
  if (d != kHeadDim) return fail(AL_EUNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, d);
  if (p.h < 1 || p.h > 4) return fail(AL_EUNSUPPORTED, "heads per group must be in [1, 4], got %d", p.h);
  if (!p.q || !p.k_cache || !p.v_cache || (!p.out && !p.part)) return fail(AL_EINVAL, "null pointer argument");
  if (!aligned16(p.k_cache) || !aligned16(p.v_cache))
    return fail(AL_EUNSUPPORTED, "k_cache and v_cache must start on a 16-byte boundary");
  if (n_all < (p.part ? 0 : 1)) return fail(AL_EINVAL, "at least one row must be read");
  const long long total = (long long)p.B * p.G * p.C;
  if (total >= 0xffffffffLL) return fail(AL_EUNSUPPORTED, "B*G*C exceeds 2^32-1 rows");
  p.total_rows = total;
  const int hp = pad_heads(p.h);
  int cs = cluster;
  if (cs <= 0) {
    cs = 1;
    while (cs < kAutoCluster && p.B * p.G * cs < di->sms && n_all / (cs * 2) >= 64) cs <<= 1;
  }
  if (cs < 1 || cs > kMaxCluster) return fail(AL_EINVAL, "cluster must be in [1, %d], got %d", kMaxCluster, cs);
  p.rows_cap = p.mode == 0 ? std::max(1, (n_all + cs - 1) / cs) : 0;
  // the deepest pipeline that leaves room for two CTAs per SM, else the deepest that fits at all
  size_t smem = 0;
  bool fits = false;
  for (int pass = 0; pass < 2 && !fits; ++pass)
    for (int st = kStages; st >= 3 && !fits; --st) {
      smem = (size_t)engine_smem(kv_dtype, hp, st) + (size_t)p.rows_cap * 4;
      p.nstage = st;
      fits = (long long)smem <= (pass == 0 ? kHalfSmBudget : (long long)(di->max_smem_optin - kAttendStaticBytes));
    }
  if (!fits) return fail(AL_EUNSUPPORTED, "row list too long for cluster %d (%zu bytes of shared memory)", cs, smem);
  p.err = di->err;
  dim3 grid((unsigned)cs, (unsigned)(p.B * p.G), 1);
  return dispatch_attend(p, kv_dtype, hp, grid, cs, smem, stream);
}

int al_gathered_attend(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                       const void* k_cache, const void* v_cache, int kv_dtype, const int64_t* rows,
                       int B, int G, int h, int d, int C, int selected_count, float scale,
                       void* out, int cluster, void* stream) {
  if (!rows) return fail(AL_EINVAL, "null rows");
  AttendParams p = {};
  p.B = B; p.G = G; p.h = h; p.C = C; p.S = selected_count; p.mode = 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = q_main; p.q_sb = q_sb; p.q_sg = q_sg; p.q_sh = q_sh;
  p.k_cache = k_cache; p.v_cache = v_cache;
  p.rows = reinterpret_cast<const long long*>(rows);
  p.out = out;
  return run_attend(p, kv_dtype, d, selected_count, cluster, stream);
}

int al_dense_decode(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                    const void* k_cache, const void* v_cache, int kv_dtype,
                    int B, int G, int h, int d, int C, int valid_length, float scale,
                    void* out, int cluster, void* stream) {
  if (valid_length < 1 || valid_length > C)
    return fail(AL_EINVAL, "valid_length=%d must be in (0, capacity=%d]", valid_length, C);
  AttendParams p = {};
  p.B = B; p.G = G; p.h = h; p.C = C; p.L = valid_length; p.mode = 1;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = q_main; p.q_sb = q_sb; p.q_sg = q_sg; p.q_sh = q_sh;
  p.k_cache = k_cache; p.v_cache = v_cache;
  p.out = out;
  return run_attend(p, kv_dtype, d, valid_length, cluster, stream);
}

static unsigned grid_for(long long n) {
  long long g = (n + kThreads - 1) / kThreads;
  if (g > 148LL * 32) g = 148LL * 32;
  return (unsigned)(g < 1 ? 1 : g);
}

int al_project_keys(const void* k_pre, const int64_t* kp_strides, const void* wk, int idx_dtype,
                    int B, int G, int T, int d, int r, void* z_out, int C_out, int start, void* stream) {
  if (!dtype_ok(idx_dtype)) return fail(AL_EINVAL, "unknown dtype code");
  if (!k_pre || !kp_strides || !wk || !z_out) return fail(AL_EINVAL, "null pointer argument");
  if (d != kHeadDim) return fail(AL_EUNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, d);
  if (r < 1 || r > kMaxR) return fail(AL_EUNSUPPORTED, "index width r must be in [1, %d]", kMaxR);
  if (B <= 0 || G <= 0 || T < 0 || start < 0 || start + T > C_out)
    return fail(AL_EINVAL, "positions [%d, %d) do not fit capacity %d", start, start + T, C_out);
  if (T == 0) return AL_OK;
  AppendParams p = {};
  p.B = B; p.G = G; p.C = C_out; p.T = T; p.r = r; p.start = start;
  p.zT = z_out; p.k_pre = k_pre; p.wk = wk;
  for (int i = 0; i < 4; ++i) p.kp_s[i] = kp_strides[i];
  dim3 grid((unsigned)((T + 31) / 32), (unsigned)(B * G), 1);
  if (idx_dtype == AL_F32) project_keys_kernel<float><<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  else project_keys_kernel<__nv_bfloat16><<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return plain_launch_check("project_keys_kernel");
}

int al_append_kvz(void* k_cache, void* v_cache, int kv_dtype,
                  const void* k_new, const int64_t* k_strides, const void* v_new, const int64_t* v_strides,
                  int new_dtype, void* zT, int idx_dtype, const void* z_new, const int64_t* z_strides,
                  const void* k_pre, const int64_t* kp_strides, const void* wk,
                  int B, int G, int C, int d, int r, int start, int T, void* stream) {
  if (!dtype_ok(kv_dtype) || !dtype_ok(new_dtype)) return fail(AL_EINVAL, "unknown dtype code");
  if (!k_cache || !v_cache || !k_new || !v_new || !k_strides || !v_strides) return fail(AL_EINVAL, "null pointer argument");
  if (d != kHeadDim) return fail(AL_EUNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, d);
  if (B <= 0 || G <= 0 || T < 0) return fail(AL_EINVAL, "bad shape");
  if (start < 0 || start + T > C) return fail(AL_ESTATE, "cache capacity %d exceeded: valid %d + new %d", C, start, T);
  if (T == 0) return AL_OK;
  AppendParams p = {};
  p.B = B; p.G = G; p.C = C; p.T = T; p.r = r; p.start = start;
  p.k_cache = k_cache; p.v_cache = v_cache; p.k_new = k_new; p.v_new = v_new;
  for (int i = 0; i < 4; ++i) { p.kn_s[i] = k_strides[i]; p.vn_s[i] = v_strides[i]; }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = grid_for((long long)B * G * T * kHeadDim);
  if (kv_dtype == AL_BF16 && new_dtype == AL_BF16) append_kv_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, kThreads, 0, st>>>(p);
  else if (kv_dtype == AL_BF16) append_kv_kernel<__nv_bfloat16, float><<<grid, kThreads, 0, st>>>(p);
  else if (new_dtype == AL_BF16) append_kv_kernel<float, __nv_bfloat16><<<grid, kThreads, 0, st>>>(p);
  else append_kv_kernel<float, float><<<grid, kThreads, 0, st>>>(p);
  int rc = plain_launch_check("append_kv_kernel");
  if (rc) return rc;
  if (z_new || k_pre) {
    if (!zT || !dtype_ok(idx_dtype)) return fail(AL_ESTATE, "this cache was created without an index table");
    if (r < 1 || r > kMaxR) return fail(AL_EUNSUPPORTED, "index width r must be in [1, %d]", kMaxR);
    p.zT = zT;
    if (z_new) {
      if (!z_strides) return fail(AL_EINVAL, "null z strides");
      p.z_new = z_new;
      for (int i = 0; i < 4; ++i) p.zn_s[i] = z_strides[i];
      const unsigned gz = grid_for((long long)B * G * r * T);
      if (idx_dtype == AL_F32) append_z_copy_kernel<float, float><<<gz, kThreads, 0, st>>>(p);
      else append_z_copy_kernel<__nv_bfloat16, __nv_bfloat16><<<gz, kThreads, 0, st>>>(p);
      return plain_launch_check("append_z_copy_kernel");
    }
    if (!wk || !kp_strides) return fail(AL_EINVAL, "k_pre given without wk or strides");
    return al_project_keys(k_pre, kp_strides, wk, idx_dtype, B, G, T, d, r, zT, C, start, stream);
  }
  return AL_OK;
}

int al_project_queries(const void* q_pre, const int64_t* qp_strides, const void* wq_t, int idx_dtype,
                       int B, int G, int h, int T, int d, int r, void* u_out, int out_f32, void* stream) {
  if (!dtype_ok(idx_dtype)) return fail(AL_EINVAL, "unknown dtype code");
  if (!q_pre || !qp_strides || !wq_t || !u_out) return fail(AL_EINVAL, "null pointer argument");
  if (d != kHeadDim) return fail(AL_EUNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, d);
  if (r < 1 || r > kMaxR) return fail(AL_EUNSUPPORTED, "index width r must be in [1, %d]", kMaxR);
  if (B <= 0 || G <= 0 || h <= 0 || T <= 0) return fail(AL_EINVAL, "bad shape");
  IndexParams p = {};
  p.B = B; p.G = G; p.h = h; p.T = T; p.r = r;
  p.q_pre = q_pre; p.wq_t = wq_t; p.out = u_out; p.out_f32 = out_f32 ? 1 : 0;
  for (int i = 0; i < 5; ++i) p.qp_s[i] = qp_strides[i];
  const unsigned grid = (unsigned)(B * G * T);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (idx_dtype == AL_F32) project_queries_kernel<float><<<grid, kThreads, 0, st>>>(p);
  else project_queries_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(p);
  return plain_launch_check("project_queries_kernel");
}

int al_candidate_scores(const void* u, const int64_t* u_strides, const void* zT, int idx_dtype,
                        int B, int G, int T, int r, int C, int lo, int hi, void* out, int out_f32, void* stream) {
  if (!dtype_ok(idx_dtype)) return fail(AL_EINVAL, "unknown dtype code");
  if (!u || !u_strides || !zT || !out) return fail(AL_EINVAL, "null pointer argument");
  if (r < 1 || r > kMaxR) return fail(AL_EUNSUPPORTED, "index width r must be in [1, %d]", kMaxR);
  if (B <= 0 || G <= 0 || T <= 0) return fail(AL_EINVAL, "bad shape");
  if (!(0 <= lo && lo <= hi && hi <= C)) return fail(AL_EINVAL, "need 0 <= lo <= hi <= C");
  if (hi == lo) return AL_OK;
  IndexParams p = {};
  p.B = B; p.G = G; p.T = T; p.r = r; p.C = C; p.lo = lo; p.hi = hi;
  p.u = u; p.zT = zT; p.out = out; p.out_f32 = out_f32 ? 1 : 0;
  for (int i = 0; i < 4; ++i) p.u_s[i] = u_strides[i];
  dim3 grid((unsigned)((hi - lo + kThreads - 1) / kThreads), (unsigned)(B * G * T), 1);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (idx_dtype == AL_F32) candidate_scores_kernel<float><<<grid, kThreads, 0, st>>>(p);
  else candidate_scores_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(p);
  return plain_launch_check("candidate_scores_kernel");
}


int al_context_local_topk(const void* q_pre, int64_t qp_sb, int64_t qp_sg, int64_t qp_sh,
                          void* zT, const void* wq_t, const void* wk, int idx_dtype,
                          const void* k_pre_new, int64_t kn_sb, int64_t kn_sg,
                          const int64_t* fixed_rows, const int64_t* off_lo,
                          int B, int G, int h, int r, int C, int lo, int hi, int k, int fixed_count, int write_col,
                          int64_t key_pos, int key_stride, int64_t* rows_out, uint64_t* keys_out, int cluster,
                          void* stream) {
  if (!rows_out || !keys_out) return fail(AL_EINVAL, "rows_out and keys_out are required");
  DecodeParams p = {};
  p.B = B; p.G = G; p.h = h; p.r = r; p.C = C;
  p.lo = lo; p.hi = hi; p.k = k; p.S = fixed_count + k; p.F = fixed_count; p.write_col = write_col;
  p.q_pre = q_pre; p.qp_sb = qp_sb; p.qp_sg = qp_sg; p.qp_sh = qp_sh;
  p.wq_t = wq_t; p.wk = wk;
  p.k_new = k_pre_new; p.kn_sb = kn_sb; p.kn_sg = kn_sg;
  p.zT = zT;
  p.fixed_rows = reinterpret_cast<const long long*>(fixed_rows);
  p.off_lo = reinterpret_cast<const long long*>(off_lo);
  p.rows_out = reinterpret_cast<long long*>(rows_out);
  p.keys_out = reinterpret_cast<unsigned long long*>(keys_out);
  p.key_pos = key_pos; p.kst = key_stride;
  if (p.S < 1) return fail(AL_EINVAL, "a shard with no rows takes no part in the step (fixed_count + k == 0)");
  return run_fused(p, AL_BF16, idx_dtype, kHeadDim, cluster, stream, false);
}

int al_context_threshold(const uint64_t* keys, int world, int rank, int B, int G, int key_stride, int k,
                         int fixed_count, int k_local, const int64_t* rows_in, int64_t* rows_attend, void* stream) {
  if (!keys || !rows_in || !rows_attend) return fail(AL_EINVAL, "null pointer argument");
  if (world < 1 || rank < 0 || rank >= world) return fail(AL_EINVAL, "rank %d outside [0, world=%d)", rank, world);
  if (B <= 0 || G <= 0 || B * (long long)G > 0x7fffffffLL) return fail(AL_EINVAL, "B and G must be positive");
  if (k < 1 || key_stride < 1 || k > (long long)world * key_stride)
    return fail(AL_EINVAL, "k=%d must lie in [1, world*key_stride=%lld]", k, (long long)world * key_stride);
  if (k_local < 0 || k_local > key_stride || fixed_count < 0)
    return fail(AL_EINVAL, "k_local=%d must lie in [0, key_stride=%d]", k_local, key_stride);
  if (fixed_count + k_local == 0) return AL_OK;
  CtxParams p = {};
  p.P = world; p.B = B; p.G = G; p.kst = key_stride; p.k = k; p.rank = rank; p.F = fixed_count; p.k_local = k_local;
  p.keys = reinterpret_cast<const unsigned long long*>(keys);
  p.rows_in = reinterpret_cast<const long long*>(rows_in);
  p.rows_attend = reinterpret_cast<long long*>(rows_attend);
  context_threshold_kernel<<<B * G, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return plain_launch_check("context_threshold_kernel");
}

int al_gathered_attend_partial(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                               const void* k_cache, const void* v_cache, int kv_dtype, const int64_t* rows,
                               int B, int G, int h, int d, int C, int n_rows, float scale,
                               float* part, int cluster, void* stream) {
  if ((!rows && n_rows > 0) || !part) return fail(AL_EINVAL, "null rows or part");
  if (n_rows < 0) return fail(AL_EINVAL, "n_rows must be >= 0");
  AttendParams p = {};
  p.B = B; p.G = G; p.h = h; p.C = C; p.S = n_rows; p.mode = 0; p.skip_neg = 1;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = q_main; p.q_sb = q_sb; p.q_sg = q_sg; p.q_sh = q_sh;
  p.k_cache = k_cache; p.v_cache = v_cache;
  p.rows = reinterpret_cast<const long long*>(rows);
  p.part = part;
  return run_attend(p, kv_dtype, d, n_rows, n_rows == 0 ? 1 : cluster, stream);
}

int al_lse_merge(const float* parts, int world, int B, int G, int h, int d, void* out, int out_dtype, void* stream) {
  if (!parts || !out) return fail(AL_EINVAL, "null pointer argument");
  if (!dtype_ok(out_dtype)) return fail(AL_EINVAL, "unknown dtype code");
  if (d != kHeadDim) return fail(AL_EUNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, d);
  if (world < 1 || B <= 0 || G <= 0 || h <= 0) return fail(AL_EINVAL, "world, B, G and h must be positive");
  const long long n = (long long)B * G * h;
  if (n * kHeadDim > 0x7fffffffLL) return fail(AL_EUNSUPPORTED, "B*G*h too large");
  const unsigned grid = (unsigned)((n * kHeadDim + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (out_dtype == AL_BF16) lse_merge_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(parts, world, (int)n, static_cast<__nv_bfloat16*>(out));
  else lse_merge_kernel<float><<<grid, 256, 0, st>>>(parts, world, (int)n, static_cast<float*>(out));
  return plain_launch_check("lse_merge_kernel");
}

int al_xchg_create(size_t bytes, void** region, void* handle_out) {
  if (!region || !handle_out || bytes == 0) return fail(AL_EINVAL, "null pointer or empty region");
  *region = nullptr;
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(exchange region)");
  if ((e = cudaMemset(ptr, 0, bytes)) != cudaSuccess) { cudaFree(ptr); return cuda_fail(e, "cudaMemset(exchange region)"); }
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, ptr)) != cudaSuccess) { cudaFree(ptr); return cuda_fail(e, "cudaIpcGetMemHandle"); }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  *region = ptr;
  return AL_OK;
}

int al_xchg_open(const void* handle, void** peer_region) {
  if (!handle || !peer_region) return fail(AL_EINVAL, "null pointer argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *peer_region = ptr;
  return AL_OK;
}

int al_xchg_close(void* peer_region) {
  if (!peer_region) return AL_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_region);
  return e == cudaSuccess ? AL_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int al_xchg_destroy(void* region) {
  if (!region) return AL_OK;
  const cudaError_t e = cudaFree(region);
  return e == cudaSuccess ? AL_OK : cuda_fail(e, "cudaFree(exchange region)");
}

int al_xchg_push(const void* src, size_t bytes, void* const* dst, int world, int rank, unsigned* done,
                 unsigned* counter, unsigned* const* peer_flags, void* stream) {
  if (!src || !dst || !done || !counter || !peer_flags) return fail(AL_EINVAL, "null pointer argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return fail(AL_EINVAL, "rank %d outside [0, world=%d)", rank, world);
  if (bytes == 0 || bytes % 16 || (reinterpret_cast<uintptr_t>(src) & 15))
    return fail(AL_EUNSUPPORTED, "the pushed data must be a positive multiple of 16 bytes starting on a 16-byte boundary");
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  XchgPush x{};
  x.src = static_cast<const int4*>(src); x.n16 = (long long)(bytes / 16);
  x.dst = reinterpret_cast<int4* const*>(dst); x.P = world; x.rank = rank;
  x.done = done; x.counter = counter; x.peer_flags = peer_flags;
  const long long blocks = std::min<long long>((x.n16 + 255) / 256, 4LL * di->sms);
  xchg_push_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x);
  return plain_launch_check("xchg_push_kernel");
}

int al_context_threshold_peer(const uint64_t* gather, const unsigned* flags, const unsigned* counter, int spin,
                              int world, int rank, int B, int G, int key_stride, int k, int fixed_count, int k_local,
                              const int64_t* rows_in, int64_t* rows_attend, void* stream) {
  if (!gather || !flags || !counter || !rows_in || !rows_attend) return fail(AL_EINVAL, "null pointer argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return fail(AL_EINVAL, "rank %d outside [0, world=%d)", rank, world);
  if (spin < 1) return fail(AL_EINVAL, "spin must be positive");
  if (B <= 0 || G <= 0 || B * (long long)G > 0x7fffffffLL) return fail(AL_EINVAL, "B and G must be positive");
  if (k < 1 || key_stride < 1 || k > (long long)world * key_stride)
    return fail(AL_EINVAL, "k=%d must lie in [1, world*key_stride=%lld]", k, (long long)world * key_stride);
  if (k_local < 0 || k_local > key_stride || fixed_count < 0)
    return fail(AL_EINVAL, "k_local=%d must lie in [0, key_stride=%d]", k_local, key_stride);
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  CtxParams p = {};
  p.P = world; p.B = B; p.G = G; p.kst = key_stride; p.k = k; p.rank = rank; p.F = fixed_count; p.k_local = k_local;
  p.keys = reinterpret_cast<const unsigned long long*>(gather);
  p.rows_in = reinterpret_cast<const long long*>(rows_in);
  p.rows_attend = reinterpret_cast<long long*>(rows_attend);
  p.wait = XchgWait{flags, counter, world, rank, spin, di->err};
  context_threshold_kernel<<<B * G, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return plain_launch_check("context_threshold_kernel");
}

int al_lse_merge_peer(const float* gather, const unsigned* flags, const unsigned* counter, int spin, int world,
                      int rank, int B, int G, int h, int d, void* out, int out_dtype, void* stream) {
  if (!gather || !flags || !counter || !out) return fail(AL_EINVAL, "null pointer argument");
  if (!dtype_ok(out_dtype)) return fail(AL_EINVAL, "unknown dtype code");
  if (d != kHeadDim) return fail(AL_EUNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, d);
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return fail(AL_EINVAL, "rank %d outside [0, world=%d)", rank, world);
  if (spin < 1) return fail(AL_EINVAL, "spin must be positive");
  if (B <= 0 || G <= 0 || h <= 0) return fail(AL_EINVAL, "B, G and h must be positive");
  const long long n = (long long)B * G * h;
  if (n * kHeadDim > 0x7fffffffLL) return fail(AL_EUNSUPPORTED, "B*G*h too large");
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  const XchgWait w{flags, counter, world, rank, spin, di->err};
  const unsigned grid = (unsigned)((n * kHeadDim + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (out_dtype == AL_BF16) lse_merge_wait_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(gather, w, (int)n, static_cast<__nv_bfloat16*>(out));
  else lse_merge_wait_kernel<float><<<grid, 256, 0, st>>>(gather, w, (int)n, static_cast<float*>(out));
  return plain_launch_check("lse_merge_wait_kernel");
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------ no-allocation entry
// Scratch of al_context_threshold_noalloc: the ranks' keys gathered into one array on this GPU. It is part of the
// library image, so every GPU that loads the library holds these 4 MiB until the process exits; no call allocates.
constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;
static __device__ __align__(256) unsigned long long g_noalloc_keys[kNoAllocScratchBytes / 8];

namespace {

// Device address of g_noalloc_keys on the current device (the host-side symbol is only a stand-in), looked up once per
// device with that device current.
unsigned long long* g_noalloc_addr[64];

int noalloc_scratch(unsigned long long** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(AL_ECUDA, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_noalloc_addr[dev]) {
    void* ptr = nullptr;
    if ((e = cudaGetSymbolAddress(&ptr, g_noalloc_keys)) != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    g_noalloc_addr[dev] = static_cast<unsigned long long*>(ptr);
  }
  *out = g_noalloc_addr[dev];
  return AL_OK;
}

// dst[q * per_rank + i] = src[q][i]: rank q's keys [B, G, key_stride] into slot q of the scratch.
__global__ void __launch_bounds__(256) gather_rank_keys_kernel(const unsigned long long* const* src, int P,
                                                                long long per_rank, unsigned long long* dst) {
  const long long n = (long long)P * per_rank, stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    const int q = (int)(i / per_rank);
    dst[i] = src[q][i - (long long)q * per_rank];
  }
}

}  // namespace

extern "C" {

int al_context_threshold_noalloc(const uint64_t* const* rank_keys, int world, int rank, int B, int G, int key_stride,
                                 int k, int fixed_count, int k_local, const int64_t* rows_in, int64_t* rows_attend,
                                 void* stream) {
  if (!rank_keys || !rows_in || !rows_attend) return fail(AL_EINVAL, "null pointer argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return fail(AL_EINVAL, "rank %d outside [0, world=%d)", rank, world);
  if (B <= 0 || G <= 0 || B * (long long)G > 0x7fffffffLL) return fail(AL_EINVAL, "B and G must be positive");
  if (k < 1 || key_stride < 1 || k > (long long)world * key_stride)
    return fail(AL_EINVAL, "k=%d must lie in [1, world*key_stride=%lld]", k, (long long)world * key_stride);
  if (k_local < 0 || k_local > key_stride || fixed_count < 0)
    return fail(AL_EINVAL, "k_local=%d must lie in [0, key_stride=%d]", k_local, key_stride);
  const long long per_rank = (long long)B * G * key_stride;
  if ((unsigned long long)world * (unsigned long long)per_rank > kNoAllocScratchBytes / 8)
    return fail(AL_EUNSUPPORTED, "world*B*G*key_stride = %lld keys exceeds the %zu keys of the no-allocation scratch",
                (long long)world * per_rank, kNoAllocScratchBytes / 8);
  if (fixed_count + k_local == 0) return AL_OK;
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  unsigned long long* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long n = (long long)world * per_rank;
  const long long blocks = std::min<long long>((n + 255) / 256, 4LL * di->sms);
  gather_rank_keys_kernel<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const unsigned long long* const*>(rank_keys),
                                                            world, per_rank, scratch);
  if ((rc = plain_launch_check("gather_rank_keys_kernel"))) return rc;
  CtxParams p = {};
  p.P = world; p.B = B; p.G = G; p.kst = key_stride; p.k = k; p.rank = rank; p.F = fixed_count; p.k_local = k_local;
  p.keys = scratch;
  p.rows_in = reinterpret_cast<const long long*>(rows_in);
  p.rows_attend = reinterpret_cast<long long*>(rows_attend);
  context_threshold_kernel<<<B * G, kThreads, 0, st>>>(p);
  return plain_launch_check("context_threshold_kernel");
}

int al_prefill_score_topk(const void* u, long long u_sh, long long u_st, const void* zT, long long z_sh, long long z_ld,
                          int H, int T, int C, int r, int q_pos0, int k, int kcap, int* idx_out, float* scores_out,
                          void* stream) {
  if (!u || !zT || !idx_out) return fail(AL_EINVAL, "null pointer argument");
  if (r != kPfR) return fail(AL_EUNSUPPORTED, "index dimension r must be %d, got %d", kPfR, r);
  if (H <= 0 || T <= 0 || C <= 0) return fail(AL_EINVAL, "H, T and C must be positive");
  if (H > 65535 || (T + kPfRows - 1) / kPfRows > 65535) return fail(AL_EUNSUPPORTED, "at most 65535 heads and 65535 row tiles");
  if (q_pos0 < 0) return fail(AL_EINVAL, "negative first query position");
  if ((long long)q_pos0 + T > C) return fail(AL_EINVAL, "query positions [%d, %lld) exceed the table's %d columns", q_pos0,
                                             (long long)q_pos0 + T, C);
  if ((long long)q_pos0 + T > 65536) return fail(AL_EUNSUPPORTED, "legal lengths above 65536 are not supported");
  if (k < 0 || kcap < k) return fail(AL_EINVAL, "need 0 <= k <= kcap (k=%d, kcap=%d)", k, kcap);
  // a row never has more candidates than its legal length (at most 65536 here), so larger slots could never be filled
  if (kcap > C || kcap > 65536) return fail(AL_EINVAL, "kcap=%d exceeds min(C=%d, 65536)", kcap, C);
  if (C % 8 || z_ld % 8 || z_sh % 8 || (reinterpret_cast<uintptr_t>(zT) & 15))
    return fail(AL_EUNSUPPORTED, "zT needs 16-byte aligned rows (C, row and head strides multiples of 8)");
  if (z_ld < C || u_st < kPfR) return fail(AL_EINVAL, "strides smaller than the rows they step over");
  if (u_st % 2 || u_sh % 2 || (reinterpret_cast<uintptr_t>(u) & 3)) return fail(AL_EUNSUPPORTED, "u needs 4-byte aligned rows");
  if (reinterpret_cast<uintptr_t>(scores_out) & 15) return fail(AL_EUNSUPPORTED, "scores_out must start on a 16-byte boundary");
  DeviceInfo* di = nullptr;
  int rc = device_info(&di);
  if (rc) return rc;
  CUtensorMap zmap;
  if (!pf_tensor_map(zT, H, C, z_sh, z_ld, &zmap)) return fail(AL_ECUDA, "cuTensorMapEncodeTiled refused the zT layout");
  rc = prepare_kernel(prefill_topk_kernel, kPfSmem, 1);
  if (rc) return rc;
  PrefillParams p{};
  p.u = static_cast<const __nv_bfloat16*>(u); p.u_sh = u_sh; p.u_st = u_st;
  p.T = T; p.C = C; p.q_pos0 = q_pos0; p.k = k; p.kcap = kcap; p.idx = idx_out; p.scores = scores_out;
  p.err = di->err;
  const dim3 grid((unsigned)H, (unsigned)((T + kPfRows - 1) / kPfRows));
  prefill_topk_kernel<<<grid, kPfThreads, kPfSmem, static_cast<cudaStream_t>(stream)>>>(p, zmap);
  return plain_launch_check("prefill_topk_kernel");
}

}  // extern "C"
