// Batched prefill scorer (config C5): for every query position p of a prefill chunk and every KV head, the indexer
// scores s[p, c] = u[p] . zT[:, c] over the candidates of a decode step at legal length p + 1 (selection.py:71-79:
// [min(4, L), max(prefix, L - 64))) and the top min(k, M(p)) of them under (score desc, position asc), the rule of
// decode.py:86-93 applied to every query row of the chunk at once. The reference selects nothing in prefill
// (qwen_wrap.py:287-289); this is the batched form of its decode-time selection.
//
// One CTA serves 16 query rows of one head (one m16 tile) and sweeps the columns its rows can see in tiles of
// 128: the zT tile is staged in shared memory by cp.async, each warp computes 16 rows x 16 columns of fp32 scores
// with bf16 mma.sync (K = 32: two k-steps), and turns them into order-preserving uint32 keys. Keys are never
// stored; each sweep recomputes them (the MMA is deterministic, so every sweep sees the same keys):
//   sweep 0: per-row histogram of the top 11 key bits        -> pivot bin, how many above it
//   sweep 1: histogram of bits 20..10 of keys in that bin     -> skipped for rows already resolved
//   sweep 2: histogram of bits 9..0                           -> skipped for rows already resolved
//   sweep 3: emission: keys above the pivot prefix, plus the first `need` keys equal to it in position order,
//            written in ascending position order.
// A row is resolved once its pivot bin holds exactly the keys it still needs (usual after sweep 1 for continuous
// scores); rows with M(p) <= k take every candidate and skip the histogram sweeps.
#pragma once
#include "al_common.cuh"

namespace al {

constexpr int kPfRows = 16;          // query rows per CTA
constexpr int kPfCols = 128;         // columns per tile
constexpr int kPfR = 32;             // index dimension r
constexpr int kPfRowPad = kPfCols + 8;   // padded tile row (bf16): ldmatrix rows land in distinct banks
constexpr int kPfBins = 2048;        // 11-bit digits; packed two 16-bit counters per word
constexpr int kPfHistWords = kPfRows * kPfBins / 2;
constexpr int kPfStages = 4;         // zT tiles in flight: three ahead of the one being scored
constexpr size_t kPfTileBytes = (size_t)kPfR * kPfRowPad * 2;
constexpr size_t kPfSmem = (size_t)kPfHistWords * 4 + kPfStages * kPfTileBytes + 2 * kPfRows * 4 * 4;

struct PrefillParams {
  const __nv_bfloat16* u;      // [H, T, 32]
  long long u_sh, u_st;        // element strides of head and row
  const __nv_bfloat16* zT;     // [H, 32, C]
  long long z_sh, z_ld;        // element strides of head and index row
  int T, C, q_pos0, k, kcap;
  int* idx;                    // [H, T, kcap] positions, ascending, -1 past the row's count
  float* scores;               // optional [H, T, C] fp32 (candidate columns only)
};

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(smem)), "l"(gmem),
               "r"(valid ? 16 : 0) : "memory");
}

__device__ __forceinline__ uint32_t pf_count(const uint32_t* h, int bin) {
  return (h[bin >> 1] >> ((bin & 1) << 4)) & 0xffffu;
}

// Pivot of one row's histogram (one warp): the bin b with (count above b) < need <= (count at or above b).
__device__ __forceinline__ void pf_pivot(const uint32_t* h, int nbins, uint32_t need, int lane, uint32_t& bin,
                                         uint32_t& above, uint32_t& in_bin) {
  const int per = nbins / 32;
  const int top = nbins - per * lane;            // lane 0 covers the highest bins
  uint32_t sum = 0;
  for (int i = top - per; i < top; i += 2) {
    const uint32_t w = h[i >> 1];
    sum += (w & 0xffffu) + (w >> 16);
  }
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const uint32_t excl = incl - sum;
  const unsigned hit = __ballot_sync(0xffffffffu, excl < need && incl >= need);
  const int src = hit ? __ffs(hit) - 1 : 0;
  uint32_t b = 0, a = 0, c = 0;
  if (lane == src) {
    uint32_t acc = excl;
    for (int i = top - 1; i >= top - per; --i) {
      const uint32_t n = pf_count(h, i);
      if (acc + n >= need) { b = (uint32_t)i; a = acc; c = n; break; }
      acc += n;
    }
  }
  bin = __shfl_sync(0xffffffffu, b, src);
  above = __shfl_sync(0xffffffffu, a, src);
  in_bin = __shfl_sync(0xffffffffu, c, src);
}

__global__ void __launch_bounds__(kThreads, 2) prefill_topk_kernel(PrefillParams p) {
  extern __shared__ __align__(128) unsigned char pf_smem[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(pf_smem);
  __nv_bfloat16* tiles = reinterpret_cast<__nv_bfloat16*>(pf_smem + (size_t)kPfHistWords * 4);
  uint32_t* m_gt = reinterpret_cast<uint32_t*>(pf_smem + (size_t)kPfHistWords * 4 + kPfStages * kPfTileBytes);
  uint32_t* m_eq = m_gt + kPfRows * 4;
  __shared__ int s_lo[kPfRows], s_hi[kPfRows], s_shift[kPfRows], s_eqb[kPfRows], s_outb[kPfRows];
  __shared__ uint32_t s_pref[kPfRows], s_need[kPfRows];
  __shared__ int s_state[kPfRows];   // 0 no candidates or taken whole; 1 refining; 2 resolved
  __shared__ int s_any;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int head = blockIdx.y;
  const int tile_row = (int)gridDim.x - 1 - (int)blockIdx.x;     // the longest rows start first
  const int t0 = tile_row * kPfRows;
  const __nv_bfloat16* zT = p.zT + (size_t)head * p.z_sh;

  if (tid < kPfRows) {
    const int t = t0 + tid;
    int lo = 0, hi = 0, kk = 0;
    if (t < p.T) {
      const int L = p.q_pos0 + t + 1;
      lo = min(4, L);
      hi = max(lo, L - 64);
      kk = min(p.k, hi - lo);
    }
    s_lo[tid] = lo; s_hi[tid] = hi;
    s_eqb[tid] = 0; s_outb[tid] = 0;
    const bool whole = kk == hi - lo;          // every candidate is taken (or there are none)
    s_state[tid] = (whole || kk == 0) ? 0 : 1;
    // whole rows: every key is above prefix 0; k = 0 rows: no key is above 0xffffffff
    s_pref[tid] = (kk == 0 && !whole) ? 0xffffffffu : 0u;
    s_need[tid] = (whole || kk == 0) ? 0u : (uint32_t)kk;
    s_shift[tid] = 0;
  }
  for (int i = tid; i < kPfHistWords; i += kThreads) hist[i] = 0;
  for (int i = tid; i < 2 * kPfRows * 4; i += kThreads) m_gt[i] = 0;
  // -1 past each row's count
  for (int i = tid; i < kPfRows * p.kcap; i += kThreads) {
    const int r = i / p.kcap, j = i - r * p.kcap, t = t0 + r;
    if (t < p.T) {
      const int L = p.q_pos0 + t + 1, lo = min(4, L), hi = max(lo, L - 64);
      if (j >= min(p.k, hi - lo)) p.idx[((size_t)head * p.T + t) * p.kcap + j] = -1;
    }
  }
  __syncthreads();

  int col_end = 0;
#pragma unroll 1
  for (int r = 0; r < kPfRows; ++r) col_end = max(col_end, s_hi[r]);
  const int ntiles = (col_end + kPfCols - 1) / kPfCols;

  // A fragments of the 16 query rows (rows past T are zero)
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t a[2][4];
  {
    const __nv_bfloat16* u = p.u + (size_t)head * p.u_sh;
    const int r0 = t0 + g, r1 = t0 + g + 8;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const int kc = ks * 16 + 2 * t4;
      a[ks][0] = r0 < p.T ? *reinterpret_cast<const uint32_t*>(u + (size_t)r0 * p.u_st + kc) : 0u;
      a[ks][1] = r1 < p.T ? *reinterpret_cast<const uint32_t*>(u + (size_t)r1 * p.u_st + kc) : 0u;
      a[ks][2] = r0 < p.T ? *reinterpret_cast<const uint32_t*>(u + (size_t)r0 * p.u_st + kc + 8) : 0u;
      a[ks][3] = r1 < p.T ? *reinterpret_cast<const uint32_t*>(u + (size_t)r1 * p.u_st + kc + 8) : 0u;
    }
  }

  auto load_tile = [&](int ti, int buf) {
    const int c0 = ti * kPfCols;
    __nv_bfloat16* dst = tiles + (size_t)buf * kPfR * kPfRowPad;
#pragma unroll
    for (int j = tid; j < kPfR * (kPfCols / 8); j += kThreads) {
      const int row = j >> 4, ch = j & 15, c = c0 + ch * 8;
      const bool ok = c + 8 <= p.C;
      cp_async16_zfill(dst + row * kPfRowPad + ch * 8, ok ? (const void*)(zT + (size_t)row * p.z_ld + c) : (const void*)zT,
                       ok);
    }
    cp_async_commit();
  };

  // sweeps 0..2 build histograms; sweep 3 emits
#pragma unroll 1
  for (int sweep = 0; sweep < 4; ++sweep) {
    if (sweep < 3) {
      if (tid == 0) {
        int any = 0;
        for (int r = 0; r < kPfRows; ++r) any |= s_state[r] == 1;
        s_any = any;
      }
      __syncthreads();
      if (!s_any && !(sweep == 0 && p.scores)) continue;
    }
    if (ntiles == 0) break;
    // this thread's two rows (g and g + 8), read once per sweep; tiles wholly inside every row's candidate range
    // skip the per-key range checks
    int lo2[2], hi2[2], st2[2], sh2[2];
    uint32_t pf2[2];
    bool eq2[2];
    int lo_max = 0, hi_min = 1 << 30;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rr = g + 8 * h;
      lo2[h] = s_lo[rr]; hi2[h] = s_hi[rr]; st2[h] = s_state[rr]; sh2[h] = s_shift[rr];
      pf2[h] = s_pref[rr]; eq2[h] = s_need[rr] > 0;
    }
#pragma unroll 1
    for (int r = 0; r < kPfRows; ++r) { lo_max = max(lo_max, s_lo[r]); hi_min = min(hi_min, s_hi[r]); }
    const int sh_cmp = sweep == 1 ? 21 : 10;
#pragma unroll
    for (int st = 0; st < kPfStages - 1; ++st) {
      if (st < ntiles) load_tile(st, st);
      else cp_async_commit();
    }
#pragma unroll 1
    for (int ti = 0; ti < ntiles; ++ti) {
      // one group per tile, empty past the end: tile ti is complete once at most kPfStages - 1 groups are pending
      if (ti + kPfStages - 1 < ntiles) load_tile(ti + kPfStages - 1, (ti + kPfStages - 1) % kPfStages);
      else cp_async_commit();
      cp_async_wait<kPfStages - 1>();
      __syncthreads();
      const __nv_bfloat16* buf = tiles + (size_t)(ti % kPfStages) * kPfR * kPfRowPad;
      const int c0 = ti * kPfCols;
      const bool interior = c0 >= lo_max && c0 + kPfCols <= hi_min;
      float acc[2][4];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        const int n0 = warp * 16 + nb * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(smem_addr(buf + (size_t)lane * kPfRowPad + n0), b0, b1, b2, b3);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nb][e] = 0.0f;
        mma_bf16_16816(acc[nb], a[0][0], a[0][1], a[0][2], a[0][3], b0, b1);
        mma_bf16_16816(acc[nb], a[1][0], a[1][1], a[1][2], a[1][3], b2, b3);
      }
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1;
          const int rr = g + 8 * h;
          const int cl = warp * 16 + nb * 8 + 2 * t4 + (e & 1);
          const int c = c0 + cl;
          if (!interior && (c < lo2[h] || c >= hi2[h])) continue;
          const uint32_t key = score_key(acc[nb][e]);
          if (sweep == 0) {
            if (p.scores) p.scores[((size_t)head * p.T + t0 + rr) * p.C + c] = acc[nb][e];
            if (st2[h] == 1) {
              const uint32_t d = key >> 21;
              atomicAdd(&hist[rr * (kPfBins / 2) + (d >> 1)], 1u << ((d & 1) << 4));
            }
          } else if (sweep < 3) {
            if (st2[h] == 1 && (key >> sh_cmp) == pf2[h]) {
              const uint32_t d = sweep == 1 ? (key >> 10) & 2047u : key & 1023u;
              atomicAdd(&hist[rr * (kPfBins / 2) + (d >> 1)], 1u << ((d & 1) << 4));
            }
          } else {
            const uint32_t kp = key >> sh2[h];
            if (kp > pf2[h]) atomicOr(&m_gt[rr * 4 + (cl >> 5)], 1u << (cl & 31));
            else if (kp == pf2[h] && eq2[h]) atomicOr(&m_eq[rr * 4 + (cl >> 5)], 1u << (cl & 31));
          }
        }
      }
      if (sweep == 3) {
        __syncthreads();
        // row rr = tid / 16 emits its 8-column segment sg in position order
        const int rr = tid >> 4, sg = tid & 15;
        const int w = sg >> 2, sh = (sg & 3) * 8;
        const uint32_t gt = (m_gt[rr * 4 + w] >> sh) & 0xffu, eq = (m_eq[rr * 4 + w] >> sh) & 0xffu;
        const int neq = __popc(eq);
        int eincl = neq;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, eincl, o, 16);
          if (sg >= o) eincl += t;
        }
        const int eq_before = s_eqb[rr] + eincl - neq;
        const int room = max(0, (int)s_need[rr] - eq_before);
        uint32_t take = eq;
        for (int j = 0, seen = 0; j < 8; ++j)
          if ((eq >> j) & 1u) { if (seen >= room) take &= ~(1u << j); ++seen; }
        const uint32_t chosen = gt | take;
        const int nch = __popc(chosen);
        int cincl = nch;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, cincl, o, 16);
          if (sg >= o) cincl += t;
        }
        int slot = s_outb[rr] + cincl - nch;
        const int t = t0 + rr;
        if (t < p.T) {
          int* out = p.idx + ((size_t)head * p.T + t) * p.kcap;
          for (int j = 0; j < 8; ++j)
            if ((chosen >> j) & 1u) {
              if (slot < p.kcap) out[slot] = c0 + sg * 8 + j;
              ++slot;
            }
        }
        const int etot = __shfl_sync(0xffffffffu, eincl, (lane & 16) | 15);
        const int ctot = __shfl_sync(0xffffffffu, cincl, (lane & 16) | 15);
        __syncwarp();
        if (sg == 15) { s_eqb[rr] += etot; s_outb[rr] += ctot; }
        if (sg < 4) { m_gt[rr * 4 + sg] = 0; m_eq[rr * 4 + sg] = 0; }
      }
      __syncthreads();
    }
    if (sweep < 3) {
      // one warp per row: pivot of this sweep's digit, then clear the row's histogram
#pragma unroll 1
      for (int rr = warp; rr < kPfRows; rr += kWarps) {
        if (s_state[rr] != 1) continue;
        const int nb = sweep == 2 ? 1024 : 2048;
        uint32_t bin, above, in_bin;
        pf_pivot(hist + rr * (kPfBins / 2), nb, s_need[rr], lane, bin, above, in_bin);
        if (lane == 0) {
          const uint32_t need = s_need[rr] - above;
          s_pref[rr] = sweep == 0 ? bin : (sweep == 1 ? (s_pref[rr] << 11) | bin : (s_pref[rr] << 10) | bin);
          s_shift[rr] = sweep == 0 ? 21 : (sweep == 1 ? 10 : 0);
          s_need[rr] = need;
          if (need == in_bin || sweep == 2) s_state[rr] = 2;
        }
        __syncwarp();
        for (int i = lane; i < kPfBins / 2; i += 32) hist[rr * (kPfBins / 2) + i] = 0;
      }
      __syncthreads();
    }
  }
}

}  // namespace al
