// Batched prefill scorer (config C5): for every query position p of a prefill chunk and every KV head, the indexer
// scores s[p, c] = u[p] . zT[:, c] over the candidates of a decode step at legal length p + 1 (selection.py:71-79:
// [min(4, L), max(prefix, L - 64))) and the top min(k, M(p)) of them under (score desc, position asc), the rule of
// decode.py:86-93 applied to every query row of the chunk at once. The reference selects nothing in prefill
// (qwen_wrap.py:287-289); this is the batched form of its decode-time selection.
//
// One CTA serves 128 query rows of one head: the tensor cores compute a 128 x 128 tile of scores per step
// (tcgen05.mma, kind::f16, bf16 operands from shared memory, fp32 accumulators in tensor memory), zT tiles arrive by
// TMA (128-byte swizzle, the layout the MMA reads as an N-major operand) in a 4-stage ring, and the accumulators sit in
// two 128-column TMEM buffers so the next tile is multiplied while the current one is read. Eight warps read TMEM, two
// threads per query row (TMEM lane = row): one takes columns 0-63 of every tile, the other 64-127; a ninth warp issues
// the copies and the MMAs. Scores are never stored: each sweep over the columns recomputes them (the MMA
// is deterministic, so every sweep sees the same values).
//
// Selection per row, on order-preserving integer keys of the scores:
//   histogram sweep: 128 bins of 2^19 key units (1/16 of an octave) below an anchor taken from the row's candidates
//                    in the first tile (twice their maximum), keys above it in bin 0, below the window in bin 127. The bin
//                    holding the k-th largest key becomes the row's window.
//   gather sweep:    the window's keys (at most 128) are copied to shared memory; one warp finds the exact k-th
//                    largest among them (a bitwise select), and how many keys equal to it are still to be taken.
//   emit sweep:      keys above the threshold, plus the first `need` keys equal to it, in position order (the two
//                    threads of a row swap their per-tile counts to place their positions).
// A window holding more than 128 keys is split again by a finer histogram sweep (bins of 2^12, 2^5, 1 units). While
// the row's scores are finite and the window lies above zero, the key of a score is its raw float bit pattern (an
// order-preserving integer for positive floats); rows with a NaN or infinity, a non-positive anchor, or a window that
// reaches zero switch to the canonical key (NaN above +inf, -0 = +0, negative scores ordered) and start over. Rows
// with M(p) <= k take every candidate and skip to the emit sweep.
#pragma once
#include <climits>
#include <cuda.h>
#include "al_common.cuh"

namespace al {

constexpr int kPfRows = 128;               // query rows per CTA: the MMA's M, one TMEM lane each
constexpr int kPfTile = 128;               // columns per tile: the MMA's N
constexpr int kPfR = 32;                   // index dimension r: the MMA's K (two kind::f16 steps of 16)
constexpr int kPfStages = 4;               // zT tiles in flight (even: stage reuse tracks the TMEM buffer's barrier)
constexpr int kPfRowWarps = 8;             // warps reading TMEM: two per lane quarter, two threads per query row
constexpr int kPfThreads = 32 * (kPfRowWarps + 1);
constexpr int kPfBins = 128;
constexpr int kPfFirstShift = 19;          // first histogram: bins of 2^19 key units
constexpr int kPfGather = 128;             // keys gathered per row
constexpr int kPfStaged = 256;             // staged output positions per row (k <= 256)
constexpr int kPfTmemCols = 2 * kPfTile;
constexpr uint32_t kPfStageBytes = kPfR * kPfTile * 2;               // 8 KB: two 64-column boxes of 32 rows
constexpr uint32_t kPfABytes = kPfRows * kPfR * 2;                   // 8 KB of u rows
constexpr uint32_t kPfWorkBytes = kPfRows * (kPfBins + 1) * 4;       // histogram (+ a sink bin) / gather / staging
constexpr size_t kPfSmem = 1024 + kPfStages * kPfStageBytes + kPfABytes + kPfWorkBytes;

static_assert(kPfStages % 2 == 0, "stage s is reused by the tile that reuses its TMEM buffer");
static_assert(3 * 16 * 512 <= kPfStages * kPfStageBytes, "three sets of 16 digit counters per row fit in the copy stages");
static_assert(kPfGather * kPfRows * 4 <= kPfWorkBytes && kPfStaged * kPfRows * 2 <= kPfWorkBytes, "work area");

// Row states (one thread per row).
constexpr int kPfNone = 0, kPfHist = 1, kPfGatherSt = 2, kPfEmit = 3, kPfDone = 4;

struct PrefillParams {
  const __nv_bfloat16* u;      // [H, T, 32]
  long long u_sh, u_st;        // element strides of head and row
  int T, C, q_pos0, k, kcap;
  int* idx;                    // [H, T, kcap] positions, ascending, -1 past the row's count
  float* scores;               // optional [H, T, C] fp32 (candidate columns only)
  unsigned* err;
};

// ------------------------------------------------------------------------------------------------ tcgen05 helpers
// Shared-memory matrix descriptor (sm_100): start address, leading and stride byte offsets (all >> 4), version 1,
// layout type in bits 61..63 (0 = no swizzle, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t pf_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B, A K-major, B N-major, M = 128, N = 128.
constexpr uint32_t kPfIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(kPfTile >> 3) << 17) |
                              ((uint32_t)(kPfRows >> 4) << 24);

__device__ __forceinline__ void pf_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
               ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kPfIdesc), "r"(accumulate) : "memory");
}
// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void pf_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n"
               ::"r"((uint32_t)__cvta_generic_to_shared(bar)) : "memory");
}
__device__ __forceinline__ void pf_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"((uint32_t)__cvta_generic_to_shared(bar)) : "memory");
}
// 3-D tiled bulk copy (x = column, y = index row, z = head) completing on `bar`; x * 2 bytes is a multiple of 128.
__device__ __forceinline__ void pf_tma3(uint32_t dst, const void* map, int x, int y, int z, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n"
               ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
               "r"((uint32_t)__cvta_generic_to_shared(bar)) : "memory");
}
// 32 consecutive TMEM columns of the thread's lane; the values are defined after pf_tmem_wait.
__device__ __forceinline__ void pf_tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
                 "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                 "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
               : "r"(taddr) : "memory");
}
// Wait for this thread's TMEM loads; the empty statements tie every loaded register to the wait so no use of them
// is scheduled before it.
__device__ __forceinline__ void pf_tmem_wait(uint32_t (&v)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) asm volatile("" : "+r"(v[j]));
}

// ------------------------------------------------------------------------------------------------ keys
// Canonical key (signed order): NaN above +inf, -0 = +0, negative scores below every non-negative one. On positive
// finite scores it equals the raw bit pattern, which is what rows in the fast mode use.
__device__ __forceinline__ int pf_canon(uint32_t v) {
  const float s = __uint_as_float(v);
  if (s != s) return INT_MAX;
  if (s == 0.0f) return 0;
  return (v & 0x80000000u) ? (int)(v ^ 0x7fffffffu) : (int)v;
}

struct PfRow {
  int lo, hi;            // candidate columns [lo, hi)
  int kk;                // keys to choose: min(k, hi - lo)
  int state;
  bool gen;              // canonical keys
  int need;              // keys still to choose inside the window
  int top, sh;           // histogram: bin (top - min(key, top)) >> sh, capped at 127
  int wlo, whi;          // window of keys (inclusive) that still holds the threshold
  int thr, eqleft;       // emission: keys above thr, then the first eqleft keys equal to it
  bool tie;              // eqleft is below the number of keys equal to thr
  int cnt;               // gathered keys, then emitted positions
  float sum;             // first histogram sweep, fast mode: non-finite sum = a NaN or infinity in the row
};

// Restart a row's selection in the canonical-key mode over the whole key range.
__device__ __forceinline__ void pf_restart_canonical(PfRow& r) {
  r.gen = true;
  r.state = kPfHist;
  r.need = r.kk;
  r.top = INT_MAX; r.sh = 25;          // (INT_MAX - key) >> 25 covers all 2^32 keys in 128 bins
  r.wlo = INT_MIN; r.whi = INT_MAX;
}

__device__ __forceinline__ void pf_red_add(uint32_t saddr) {
  asm volatile("red.shared.add.u32 [%0], 1;\n" ::"r"(saddr) : "memory");
}
__device__ __forceinline__ void pf_st32(uint32_t saddr, int v) {
  asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(saddr), "r"(v) : "memory");
}
__device__ __forceinline__ void pf_st16(uint32_t saddr, int v) {
  asm volatile("st.shared.u16 [%0], %1;\n" ::"r"(saddr), "h"((unsigned short)v) : "memory");
}
__device__ __forceinline__ uint32_t pf_ld32(uint32_t saddr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];\n" : "=r"(v) : "r"(saddr) : "memory");
  return v;
}
__device__ __forceinline__ int pf_ld16(uint32_t saddr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(saddr) : "memory");
  return (int)v;
}

// Per-thread pointers and roles of a row thread.
struct PfCtx {
  uint32_t tcol;        // TMEM address of the warp's lane quarter, column 0
  uint32_t hist;        // the row's bin-0 word of the histogram (bins 512 bytes apart; bin kPfBins is a sink)
  uint32_t stage;       // the row's 512-byte slot of 256 staged output positions (16-bit)
  uint32_t gbase;       // this thread's first gather slot (half 0: slot 0, half 1: slot 127; slot i of row r is word
                        // i * 128 + r of the work area)
  int gstep;            // +512 or -512 bytes per gathered key
  int* out;             // the row's output positions (used directly when k > kPfStaged)
  float* srow;          // the row's scores (optional)
  int half;             // 0: columns 0-63 of every tile, 1: columns 64-127
  int q;                // lane quarter (named barrier 2 + q pairs the row's two warps)
  int row;
  bool staged;
};

// Candidates [jlo, jhi) of a 32-column chunk as a bit mask (0 < jhi, jlo < 32).
__device__ __forceinline__ uint32_t pf_vmask(int jlo, int jhi) {
  const uint32_t hi = jhi >= 32 ? 0xffffffffu : ((1u << jhi) - 1u);
  const uint32_t lo = jlo <= 0 ? 0xffffffffu : ~((1u << jlo) - 1u);
  return hi & lo;
}

// Each sweep has one hot chunk routine (fast-mode keys, all 32 columns candidates, no ties) and one generic routine
// (canonical keys where the row uses them, a candidate mask, ties), so the code that runs per key stays small.
__device__ __forceinline__ int pf_key(uint32_t v, bool gen) { return gen ? pf_canon(v) : (int)v; }

// Predicated shared store (no branch around it).
__device__ __forceinline__ void pf_st32_if(uint32_t saddr, int v, bool p) {
  asm volatile("{\n .reg .pred q;\n setp.ne.b32 q, %2, 0;\n @q st.shared.b32 [%0], %1;\n}\n"
               ::"r"(saddr), "r"(v), "r"((int)p) : "memory");
}

// Histogram sweep, hot chunk (the row's first sweep in fast mode): every key adds one to its bin
// (top - min(key, top)) >> 19, capped at 127, one unconditional shared-memory reduction per key; the scores are summed
// in four chains to detect a NaN or an infinity.
__device__ __forceinline__ void pf_hist_hot(const uint32_t (&v)[32], PfRow& r, uint32_t hist) {
  float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int key = (int)v[j];
    a[j & 3] += __uint_as_float(v[j]);
    const unsigned d = min(((unsigned)r.top - (unsigned)min(key, r.top)) >> kPfFirstShift, (unsigned)(kPfBins - 1));
    pf_red_add(hist + (d << 9));
  }
  r.sum += (a[0] + a[1]) + (a[2] + a[3]);
}

// Histogram sweep, generic chunk: candidates vm only, keys outside the row's window go to the sink bin. `first`: the
// row's first sweep (fast-mode rows add up their scores).
__device__ __forceinline__ void pf_hist_gen(const uint32_t (&v)[32], uint32_t vm, PfRow& r, uint32_t hist, bool first) {
  float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const bool sum = first && !r.gen;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const bool valid = (vm >> j) & 1u;
    const int key = pf_key(v[j], r.gen);
    a[j & 3] += (valid && sum) ? __uint_as_float(v[j]) : 0.0f;
    unsigned d = min(((unsigned)r.top - (unsigned)min(key, r.top)) >> r.sh, (unsigned)(kPfBins - 1));
    const bool in = valid && ((unsigned)key - (unsigned)r.wlo <= (unsigned)r.whi - (unsigned)r.wlo);
    d = in ? d : (unsigned)kPfBins;
    pf_red_add(hist + (d << 9));
  }
  if (sum) r.sum += (a[0] + a[1]) + (a[2] + a[3]);
}

// Gather sweep: the window's keys go to the row's 128 slots, the lower-column thread filling them from the front and
// the other from the back (the window holds at most 128 keys, so they never meet; the count is r.cnt). Stores are
// predicated, not branched around.
template <bool HOT>
__device__ __forceinline__ void pf_gather_chunk(const uint32_t (&v)[32], uint32_t vm, PfRow& r, uint32_t base, int step) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int key = HOT ? (int)v[j] : pf_key(v[j], r.gen);
    const bool in = (HOT || ((vm >> j) & 1u)) && ((unsigned)key - (unsigned)r.wlo <= (unsigned)r.whi - (unsigned)r.wlo) &&
                    r.cnt < kPfGather;
    pf_st32_if(base + (uint32_t)(r.cnt * step), key, in);
    r.cnt += in ? 1 : 0;
  }
}

// Emit sweep: bit j of `take` for a key at or above the threshold (hot) or above it (generic, with ties in `eq`),
// limited to the candidates.
__device__ __forceinline__ void pf_emit_hot(const uint32_t (&v)[32], const PfRow& r, uint32_t& take) {
  uint32_t t = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) t |= ((int)v[j] >= r.thr ? 1u : 0u) << j;
  take = t;
}
__device__ __forceinline__ void pf_emit_gen(const uint32_t (&v)[32], uint32_t vm, const PfRow& r, uint32_t& take,
                                            uint32_t& eq) {
  uint32_t t = 0, e = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int key = pf_key(v[j], r.gen);
    t |= ((r.tie ? key > r.thr : key >= r.thr) ? 1u : 0u) << j;
    e |= (r.tie && key == r.thr ? 1u : 0u) << j;
  }
  take = t & vm;
  eq = e & vm;
}

// The n lowest set bits of m.
__device__ __forceinline__ uint32_t pf_keep_low(uint32_t m, int n) {
  uint32_t o = 0;
  while (n > 0 && m) { const uint32_t b = m & (0u - m); o |= b; m ^= b; --n; }
  return o;
}

// Largest candidate score of a chunk (candidates [jlo, jhi)), NaN ignored.
__device__ __forceinline__ float pf_chunk_max(const uint32_t (&v)[32], int jlo, int jhi) {
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j >= jlo && j < jhi) m = fmaxf(m, __uint_as_float(v[j]));
  return m;
}

// The row's anchor, from the largest score m among its candidates in the first tile: twice that. A row without a
// positive finite maximum there uses canonical keys from the start.
__device__ __forceinline__ void pf_anchor(float m, PfRow& r) {
  if (m > 0.0f && m <= 3.402823466e38f) {
    r.gen = false;
    r.top = __float_as_int(2.0f * m);
    r.sh = kPfFirstShift;
    r.wlo = INT_MIN; r.whi = INT_MAX;
    r.need = r.kk;
    r.sum = 0.0f;
  } else {
    pf_restart_canonical(r);
  }
}

// Bounded wait; after the first wait that gives up, the CTA stops waiting (its results are invalid and flagged).
__device__ __forceinline__ void pf_wait(uint64_t* bar, unsigned parity, volatile int* abort_flag, unsigned* err) {
  if (*abort_flag) return;
  if (!mbar_wait(bar, parity)) {
    *abort_flag = 1;
    atomicOr(err, kErrWaitLimit);
  }
}

// Emit sweep, end of a tile: the two threads of the row swap their counts (keys above the threshold, keys equal to
// it) through shared memory, the lower half takes its ties first, and each writes its positions in order after the
// other's when it is the upper half. Both threads keep the same running count.
__device__ __forceinline__ void pf_emit_tile(const PfCtx& c, PfRow& r, uint32_t* s_ex, int par, int cbase,
                                             uint32_t (&take)[2], uint32_t (&eq)[2]) {
  const uint32_t mine = (uint32_t)(__popc(take[0]) + __popc(take[1])) |
                        ((uint32_t)(__popc(eq[0]) + __popc(eq[1])) << 16);
  s_ex[(par * 2 + c.half) * kPfRows + c.row] = mine;
  asm volatile("bar.sync %0, 64;\n" ::"r"(2 + c.q) : "memory");
  const uint32_t xa = s_ex[(par * 2 + 0) * kPfRows + c.row], xb = s_ex[(par * 2 + 1) * kPfRows + c.row];
  const int gta = (int)(xa & 0xffffu), eqa = (int)(xa >> 16), gtb = (int)(xb & 0xffffu), eqb = (int)(xb >> 16);
  const int rem = r.eqleft > 0 ? r.eqleft : 0;
  const int alla = min(eqa, rem), allb = min(eqb, rem - alla);
  int allow = c.half ? allb : alla;
  uint32_t m0 = take[0], m1 = take[1];
  if (eq[0] | eq[1]) {
    const uint32_t e0 = pf_keep_low(eq[0], allow);
    allow -= __popc(e0);
    m0 |= e0;
    m1 |= pf_keep_low(eq[1], allow);
  }
  int slot = r.cnt + (c.half ? gta + alla : 0);
  const int cap = r.kk;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    uint32_t m = w ? m1 : m0;
    const int cb = cbase + 32 * w;
    while (m) {
      const int j = __ffs(m) - 1;
      m &= m - 1;
      if (slot < cap) {                       // always, unless the launch was flagged invalid
        if (c.staged) pf_st16(c.stage + ((uint32_t)slot << 1), cb + j);
        else c.out[slot] = cb + j;
      }
      ++slot;
    }
  }
  r.cnt += gta + alla + gtb + allb;
  r.eqleft -= alla + allb;
}

// One sweep of a row thread over nt tiles of TMEM scores (global tile counter g): this thread's two chunks of each
// tile (columns 64 * half .. + 63). Rows in state KIND do that sweep's work; in the CTA's first sweep every row with
// candidates also writes its scores when asked to.
template <int KIND>
__device__ void pf_sweep(int nt, int& g, bool first, PfRow& r, const PfCtx& c, uint64_t* tfull, uint64_t* tfree,
                         uint32_t* s_ex, volatile int* abort_flag, unsigned* err) {
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int i = 0; i < nt; ++i, ++g) {
    const int buf = g & 1;
    pf_wait(&tfull[buf], (unsigned)(g >> 1) & 1u, abort_flag, err);
    tmem_fence_after_sync();
    const int c0 = i * kPfTile;
    const bool act = r.state == KIND;
    if (KIND == kPfHist && first && i == 0) {          // the anchor: both threads of the row read the whole tile
      float m = -INFINITY;
#pragma unroll 1
      for (int w = 0; w < kPfTile / 32; ++w) {
        uint32_t v[32];
        pf_tmem_ld32(c.tcol + (uint32_t)(buf * kPfTile + 32 * w), v);
        pf_tmem_wait(v);
        m = fmaxf(m, pf_chunk_max(v, r.lo - 32 * w, r.hi - 32 * w));
      }
      if (act) pf_anchor(m, r);
    }
    uint32_t take[2] = {0u, 0u}, eq[2] = {0u, 0u};
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const int cq = c0 + 64 * c.half + 32 * w;
      uint32_t v[32];
      pf_tmem_ld32(c.tcol + (uint32_t)(buf * kPfTile + 64 * c.half + 32 * w), v);
      pf_tmem_wait(v);
      if (w == 1) {                                     // the buffer is in registers: the MMA may overwrite it
        tmem_fence_before_sync();
        __syncwarp();
        if (lane == 0) pf_arrive(&tfree[buf]);
      }
      const int jlo = r.lo - cq, jhi = r.hi - cq;      // candidates of this chunk: [jlo, jhi) clipped to [0, 32)
      if (jhi <= 0 || jlo >= 32) continue;
      const bool full = jlo <= 0 && jhi >= 32;
      const uint32_t vm = full ? 0xffffffffu : pf_vmask(jlo, jhi);
      if (first && c.srow != nullptr) {
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(c.srow + cq + j) = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                                      __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if ((vm >> j) & 1u) c.srow[cq + j] = __uint_as_float(v[j]);
        }
      }
      if (KIND == kPfNone || !act) continue;
      const bool hot = full && !r.gen;
      if (KIND == kPfHist) {
        if (hot && first) pf_hist_hot(v, r, c.hist);
        else pf_hist_gen(v, vm, r, c.hist, first);
      } else if (KIND == kPfGatherSt) {
        if (hot) pf_gather_chunk<true>(v, vm, r, c.gbase, c.gstep);
        else pf_gather_chunk<false>(v, vm, r, c.gbase, c.gstep);
      } else if (KIND == kPfEmit) {
        if (hot && !r.tie) pf_emit_hot(v, r, take[w]);
        else pf_emit_gen(v, vm, r, take[w], eq[w]);
      }
    }
    if (KIND == kPfEmit) pf_emit_tile(c, r, s_ex, g & 1, c0 + 64 * c.half, take, eq);
  }
}

// After a histogram sweep (both threads of the row, reading the same counts): the bin holding the row's need-th
// largest key (counting from the top) becomes the window. `bad`: after the row's first sweep, a fast-mode row whose
// scores did not sum to a finite value (a NaN or an infinity among them) starts over with canonical keys.
__device__ __forceinline__ void pf_after_hist(PfRow& r, uint32_t hist, bool bad) {
  unsigned cum = 0, before = 0, inb = 0;
  int piv = -1;
#pragma unroll 8
  for (int d = 0; d < kPfBins; ++d) {
    const unsigned cnt = pf_ld32(hist + ((uint32_t)d << 9));
    if (piv < 0 && cum + cnt >= (unsigned)r.need) { piv = d; before = cum; inb = cnt; }
    cum += cnt;
  }
  if (bad && !r.gen) { pf_restart_canonical(r); return; }
  if (piv < 0) { piv = kPfBins - 1; before = cum; inb = 0; }   // unreachable: the window holds the need-th key
  const long long top = r.top;
  long long hk = piv == 0 ? (long long)r.whi : top - ((long long)piv << r.sh);
  long long lk = piv == kPfBins - 1 ? (long long)r.wlo : top - ((long long)(piv + 1) << r.sh) + 1;
  hk = hk < r.whi ? hk : (long long)r.whi;
  lk = lk > r.wlo ? lk : (long long)r.wlo;
  r.need -= (int)before;
  if (!r.gen && lk <= 0) { pf_restart_canonical(r); return; }
  if (hk == lk) {                                   // a single key value: it is the threshold
    r.state = kPfEmit; r.thr = (int)hk; r.eqleft = r.need; r.tie = r.need < (int)inb; r.cnt = 0;
  } else if (inb <= (unsigned)kPfGather) {
    r.state = kPfGatherSt; r.wlo = (int)lk; r.whi = (int)hk; r.cnt = 0;
  } else {                                          // too many keys to gather: a finer histogram of the window
    const unsigned long long span = (unsigned long long)(hk - lk);
    const int bits = 64 - __clzll((long long)span);
    r.wlo = (int)lk; r.whi = (int)hk; r.top = (int)hk; r.sh = bits > 7 ? bits - 7 : 0;
  }
}

// A window whose keys overflowed a thread's gather slots: split it by a finer histogram instead.
__device__ __forceinline__ void pf_refine(PfRow& r) {
  const unsigned long long span = (unsigned long long)((long long)r.whi - (long long)r.wlo);
  const int bits = 64 - __clzll((long long)span);
  r.state = kPfHist; r.top = r.whi; r.sh = bits > 7 ? bits - 7 : 0;
}

// After a gather sweep, both threads of each row: the exact need-th largest of the gathered keys, by a radix select on
// the offsets o = whi - key, four bits per pass from the top: each thread adds its own keys that match the prefix so
// far to the row's 16 digit counters, the pair meets at a named barrier, and both pick the digit holding the need-th
// smallest offset. Counters live in the (idle) copy stages, three sets in turn so one barrier per pass suffices; the
// gathered keys are read from their slots (slot i of row r at word i * 128 + r: the 32 rows of a warp hit 32 banks).
// Then the threshold, how many keys equal to it the row takes and whether that is fewer than all of them; a row whose
// threads gathered more than 128 keys is marked for a finer histogram.
__device__ __forceinline__ void pf_resolve(const PfRow& r, const PfCtx& c, uint32_t s_work, uint32_t s_bins,
                                           const int* s_gn, uint32_t* s_ex, int* s_thr, int* s_eql, uint8_t* s_flag) {
  const bool act = r.state == kPfGatherSt;
  const int n0 = s_gn[c.row], n1 = s_gn[kPfRows + c.row];          // slots [0, n0) and [128 - n1, 128)
  const bool work = act && n0 + n1 <= kPfGather;
  const unsigned whi = (unsigned)r.whi, span = whi - (unsigned)r.wlo;
  const int bits = work ? 32 - __clz((int)(span | 1u)) : 0;
  const int npass = ((int)__reduce_max_sync(0xffffffffu, (unsigned)bits) + 3) / 4;   // the same in both warps
  const int mlo = c.half ? kPfGather - n1 : 0, mhi = c.half ? kPfGather : n0;
  const uint32_t col = s_work + (uint32_t)c.row * 4u, bins = s_bins + (uint32_t)c.row * 4u;
  unsigned pref = 0;
  int rem = r.need;
#pragma unroll 1
  for (int pass = 0; pass < npass; ++pass) {
    const int shift = 4 * (npass - 1 - pass);
    const uint32_t cur = bins + (uint32_t)(pass % 3) * (16 * 512), nxt = bins + (uint32_t)((pass + 1) % 3) * (16 * 512);
#pragma unroll
    for (int d = 0; d < 8; ++d) pf_st32(nxt + (uint32_t)(8 * c.half + d) * 512u, 0);
    if (work) {
#pragma unroll 4
      for (int i = mlo; i < mhi; ++i) {
        const unsigned o = whi - pf_ld32(col + (uint32_t)i * (kPfRows * 4));
        const bool match = shift + 4 >= 32 || ((o ^ pref) >> (shift + 4)) == 0u;
        if (match) pf_red_add(cur + (((o >> shift) & 15u) << 9));
      }
    }
    asm volatile("bar.sync %0, 64;\n" ::"r"(2 + c.q) : "memory");
    if (work) {
      unsigned cum = 0;
      int dig = 15;
#pragma unroll 1
      for (int d = 0; d < 16; ++d) {
        const unsigned n = pf_ld32(cur + (uint32_t)d * 512u);
        if (cum + n >= (unsigned)rem) { dig = d; break; }
        cum += n;
      }
      rem -= (int)cum;
      pref |= (unsigned)dig << shift;
    }
  }
  int gt = 0, eq = 0;
  if (work) {
#pragma unroll 4
    for (int i = mlo; i < mhi; ++i) {
      const unsigned o = whi - pf_ld32(col + (uint32_t)i * (kPfRows * 4));
      gt += o < pref ? 1 : 0;
      eq += o == pref ? 1 : 0;
    }
  }
  s_ex[c.half * kPfRows + c.row] = (uint32_t)gt | ((uint32_t)eq << 16);
  asm volatile("bar.sync %0, 64;\n" ::"r"(2 + c.q) : "memory");
  if (c.half == 0 && act) {
    if (!work) {
      s_flag[c.row] = 2;
    } else {
      const uint32_t x0 = s_ex[c.row], x1 = s_ex[kPfRows + c.row];
      const int gtt = (int)((x0 & 0xffffu) + (x1 & 0xffffu)), eqq = (int)((x0 >> 16) + (x1 >> 16));
      s_thr[c.row] = (int)(whi - pref);
      s_eql[c.row] = r.need - gtt;
      s_flag[c.row] = (r.need - gtt) < eqq ? 1 : 0;
    }
  }
}

// Grid (H, ceil(T / 128)), 288 threads: warps 0-7 hold two threads per query row (warp w: lane quarter w % 4, column
// half w / 4), warp 8 issues the TMA copies and the MMAs.
__global__ void __launch_bounds__(kPfThreads, 2)
    prefill_topk_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap zmap) {
  extern __shared__ __align__(1024) unsigned char pf_raw[];
  __shared__ uint64_t s_full[kPfStages], s_tfull[2], s_tfree[2];
  __shared__ uint32_t s_taddr;
  __shared__ int s_nt, s_kind, s_flags, s_maxhi[4], s_anyovf;
  __shared__ volatile int s_abort;
  __shared__ uint32_t s_ex[2 * 2 * kPfRows];          // emit: [tile parity][half][row] counts
  __shared__ int s_thr[kPfRows], s_eql[kPfRows];
  __shared__ int s_gn[2 * kPfRows];
  __shared__ uint8_t s_flag[kPfRows], s_bad[kPfRows];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int head = blockIdx.x;
  const int t0 = ((int)gridDim.y - 1 - (int)blockIdx.y) * kPfRows;      // the longest rows of every head start first
  const uint32_t raw = smem_addr(pf_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;                             // 128-byte swizzle atoms: 1 KB aligned
  const uint32_t s_stage = sb;
  const uint32_t s_a = sb + kPfStages * kPfStageBytes;
  const uint32_t s_work = s_a + kPfABytes;
  const bool row_thread = warp < kPfRowWarps;

  if (tid == 0) {
    for (int s = 0; s < kPfStages; ++s) mbar_init(&s_full[s], 1);
    for (int b = 0; b < 2; ++b) { mbar_init(&s_tfull[b], 1); mbar_init(&s_tfree[b], kPfRowWarps); }
    mbar_init_fence();
    s_abort = 0; s_flags = 0; s_anyovf = 0;
    for (int i = 0; i < 4; ++i) s_maxhi[i] = 0;
  }
  if (warp == 0) { tmem_alloc(&s_taddr, kPfTmemCols); tmem_relinquish(); }

  PfCtx c;
  c.q = warp & 3; c.half = (warp >> 2) & 1; c.row = 32 * c.q + lane;
  const int t = t0 + c.row;
  PfRow r;
  r.lo = 0; r.hi = 0; r.kk = 0; r.state = kPfNone; r.gen = false; r.need = 0; r.top = INT_MAX; r.sh = 25;
  r.wlo = INT_MIN; r.whi = INT_MAX; r.thr = INT_MIN; r.eqleft = 0; r.tie = false; r.cnt = 0; r.sum = 0.0f;
  if (row_thread) {
    if (c.half == 0) {
      // u row -> the MMA's A operand: K-major, no swizzle: 8 x (8 bf16) core matrices, K chunks 128 B apart, 8-row
      // groups 512 B apart. Rows past the chunk are zero.
#pragma unroll
      for (int kc = 0; kc < kPfR / 8; ++kc) {
        uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
        if (t < p.T) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(p.u + (size_t)head * p.u_sh + (size_t)t * p.u_st + kc * 8);
          w0 = src[0]; w1 = src[1]; w2 = src[2]; w3 = src[3];
        }
        const uint32_t dst = s_a + (uint32_t)(c.row >> 3) * 512u + (uint32_t)kc * 128u + (uint32_t)(c.row & 7) * 16u;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(dst), "r"(w0), "r"(w1), "r"(w2), "r"(w3) : "memory");
      }
      s_bad[c.row] = 0; s_flag[c.row] = 0;
    }
    for (uint32_t o = (uint32_t)tid * 16u; o < kPfWorkBytes; o += 2 * kPfRows * 16u)
      asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};\n" ::"r"(s_work + o), "r"(0) : "memory");
    if (t < p.T) {
      const int L = p.q_pos0 + t + 1;
      r.lo = min(4, L);
      r.hi = max(r.lo, L - 64);
      r.kk = min(p.k, r.hi - r.lo);
      if (r.kk == 0) r.state = kPfNone;
      else if (r.kk == r.hi - r.lo) r.state = kPfEmit;        // every candidate: thr = INT_MIN takes them all
      else r.state = kPfHist;                                  // the anchor of the first sweep sets the window
    }
  }
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");   // u rows visible to the tensor cores
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tbase = s_taddr;

  c.staged = p.k <= kPfStaged;
  c.tcol = tbase + ((uint32_t)(32 * c.q) << 16);
  c.hist = s_work + (uint32_t)c.row * 4u;
  c.stage = s_work + (uint32_t)c.row * (kPfGather * 4);
  c.gbase = s_work + (uint32_t)c.row * 4u + (c.half ? (uint32_t)(kPfGather - 1) * (kPfRows * 4) : 0u);
  c.gstep = c.half ? -(kPfRows * 4) : kPfRows * 4;
  c.out = (row_thread && t < p.T) ? p.idx + ((size_t)head * p.T + t) * p.kcap : nullptr;
  c.srow = (p.scores && row_thread && t < p.T) ? p.scores + ((size_t)head * p.T + t) * p.C : nullptr;
  const uint64_t adesc0 = pf_sdesc(s_a, 128, 512, 0);

  int g = 0;
  bool first = true;
#pragma unroll 1
  for (;;) {
    if (row_thread) {
      // the next sweep: histogram while any row needs one, then gather, then emit; its columns reach the largest
      // candidate end among the rows taking part (every row with candidates in a first sweep writing scores)
      const int want = r.state == kPfHist ? 1 : r.state == kPfGatherSt ? 2 : r.state == kPfEmit ? 4 : 0;
      const unsigned wor = __reduce_or_sync(0xffffffffu, (unsigned)want);
      const int mh1 = (int)__reduce_max_sync(0xffffffffu, (unsigned)(want == 1 ? r.hi : 0));
      const int mh2 = (int)__reduce_max_sync(0xffffffffu, (unsigned)(want == 2 ? r.hi : 0));
      const int mh4 = (int)__reduce_max_sync(0xffffffffu, (unsigned)(want == 4 ? r.hi : 0));
      const int mha = (int)__reduce_max_sync(0xffffffffu, (unsigned)r.hi);
      if (lane == 0) {
        atomicOr(&s_flags, (int)wor);
        atomicMax(&s_maxhi[0], mh1); atomicMax(&s_maxhi[1], mh2); atomicMax(&s_maxhi[2], mh4);
        atomicMax(&s_maxhi[3], mha);
      }
      asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kPfRowWarps) : "memory");
      if (tid == 0) {
        const int f = s_flags;
        const int kind = (f & 1) ? kPfHist : (f & 2) ? kPfGatherSt : (f & 4) ? kPfEmit : kPfNone;
        int mh = kind == kPfHist ? s_maxhi[0] : kind == kPfGatherSt ? s_maxhi[1] : kind == kPfEmit ? s_maxhi[2] : 0;
        if (first && p.scores) mh = max(mh, s_maxhi[3]);
        if (s_abort) mh = 0;
        s_kind = kind;
        s_nt = (mh + kPfTile - 1) / kPfTile;
        s_flags = 0;
        for (int i = 0; i < 4; ++i) s_maxhi[i] = 0;
      }
    }
    __syncthreads();
    const int nt = s_nt, kind = s_kind;
    if (nt == 0) break;
    if (!row_thread) {
      if (lane == 0) {
        // producer: TMA of zT tile gg (columns x .. x + 127 of this head) into stage gg % kPfStages, once the MMA of
        // the tile that used the stage before (gg - kPfStages, same TMEM buffer) is complete; in a new sweep those
        // MMAs finished before the row threads closed the previous one
        const int gs = g;
        auto issue = [&](int gg) {
          const int s = gg % kPfStages;
          if (gg - kPfStages >= gs)
            pf_wait(&s_tfull[(gg - kPfStages) & 1], (unsigned)((gg - kPfStages) >> 1) & 1u, &s_abort, p.err);
          mbar_arrive_expect_tx(&s_full[s], kPfStageBytes);
          const uint32_t dst = s_stage + (uint32_t)s * kPfStageBytes;
          const int x = (gg - gs) * kPfTile;
          pf_tma3(dst, &zmap, x, 0, head, &s_full[s]);
          pf_tma3(dst + kPfStageBytes / 2, &zmap, x + 64, 0, head, &s_full[s]);
        };
        for (int i = 0; i < min(nt, kPfStages - 1); ++i) issue(gs + i);
#pragma unroll 1
        for (int i = 0; i < nt; ++i) {
          const int gg = gs + i, s = gg % kPfStages, buf = gg & 1;
          pf_wait(&s_full[s], (unsigned)(gg / kPfStages) & 1u, &s_abort, p.err);
          if (gg >= 2) pf_wait(&s_tfree[buf], (unsigned)((gg >> 1) - 1) & 1u, &s_abort, p.err);
          tmem_fence_after_sync();
          const uint32_t bst = s_stage + (uint32_t)s * kPfStageBytes;
          // B: N-major, 128-byte swizzle; 64-column groups 4 KB apart, 8-row groups 1 KB apart; a K step of 16 rows
          // advances B by 2 KB and A by 256 B
#pragma unroll
          for (int ks = 0; ks < kPfR / 16; ++ks)
            pf_mma(tbase + (uint32_t)(buf * kPfTile), adesc0 + (uint64_t)((ks * 256) >> 4),
                   pf_sdesc(bst + (uint32_t)ks * 2048u, kPfStageBytes / 2, 1024, 2), ks > 0 ? 1u : 0u);
          pf_commit(&s_tfull[buf]);
          if (i + kPfStages - 1 < nt) issue(gg + kPfStages - 1);
        }
      }
      __syncwarp();
      g += nt;
    } else {
      if (kind == kPfHist) {
        pf_sweep<kPfHist>(nt, g, first, r, c, s_tfull, s_tfree, s_ex, &s_abort, p.err);
        if (first && r.state == kPfHist && !r.gen && !isfinite(r.sum)) s_bad[c.row] = 1;
        asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kPfRowWarps) : "memory");
        const bool was = r.state == kPfHist;
        if (was) pf_after_hist(r, c.hist, first && s_bad[c.row]);
        asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kPfRowWarps) : "memory");
        if (was)                                         // clear the row's bins (and its sink) for the next histogram
          for (int d = c.half * 65; d < min(kPfBins + 1, c.half * 65 + 65); ++d) pf_st32(c.hist + ((uint32_t)d << 9), 0);
      } else if (kind == kPfGatherSt) {
        pf_sweep<kPfGatherSt>(nt, g, first, r, c, s_tfull, s_tfree, s_ex, &s_abort, p.err);
        s_gn[c.half * kPfRows + c.row] = r.state == kPfGatherSt ? r.cnt : 0;
#pragma unroll
        for (int d = 0; d < 8; ++d) pf_st32(s_stage + (uint32_t)c.row * 4u + (uint32_t)(8 * c.half + d) * 512u, 0);
        if (tid == 0) s_anyovf = 0;
        asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kPfRowWarps) : "memory");
        pf_resolve(r, c, s_work, s_stage, s_gn, s_ex, s_thr, s_eql, s_flag);
        asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kPfRowWarps) : "memory");
        if (r.state == kPfGatherSt) {
          const int f = s_flag[c.row];
          if (f == 2) {
            pf_refine(r);
            s_anyovf = 1;
          } else {
            r.state = kPfEmit; r.thr = s_thr[c.row]; r.eqleft = s_eql[c.row]; r.tie = f == 1; r.cnt = 0;
          }
        }
        asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kPfRowWarps) : "memory");
        if (s_anyovf)                                    // a finer histogram follows: clear the work area
          for (uint32_t o = (uint32_t)tid * 16u; o < kPfWorkBytes; o += 2 * kPfRows * 16u)
            asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};\n" ::"r"(s_work + o), "r"(0) : "memory");
      } else if (kind == kPfEmit) {
        pf_sweep<kPfEmit>(nt, g, first, r, c, s_tfull, s_tfree, s_ex, &s_abort, p.err);
        if (r.state == kPfEmit) r.state = kPfDone;
      } else {
        pf_sweep<kPfNone>(nt, g, first, r, c, s_tfull, s_tfree, s_ex, &s_abort, p.err);
      }
    }
    first = false;
  }

  // the producer's last copies and MMAs, whatever happened to the waits above (bounded; complete already unless a wait
  // gave up): nothing may still write this CTA's shared memory or tensor memory when it exits
  if (!row_thread && lane == 0 && g > 0) {
    for (int gg = max(0, g - kPfStages); gg < g; ++gg) mbar_wait(&s_full[gg % kPfStages], (unsigned)(gg / kPfStages) & 1u);
    mbar_wait(&s_tfull[(g - 1) & 1], (unsigned)((g - 1) >> 1) & 1u);
  }
  // output rows (warp w: rows 32 q + 16 half .. + 15): the staged positions (or the ones already written), then -1
  if (row_thread) {
    asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kPfRowWarps) : "memory");
    const int n_mine = (r.state == kPfDone) ? min(r.cnt, r.kk) : 0;
#pragma unroll 1
    for (int rr = 0; rr < 16; ++rr) {
      const int ln = 16 * c.half + rr, row = 32 * c.q + ln, tr = t0 + row;
      const int n = __shfl_sync(0xffffffffu, n_mine, ln);
      if (tr >= p.T) continue;
      int* o = p.idx + ((size_t)head * p.T + tr) * p.kcap;
      const uint32_t st = s_work + (uint32_t)row * (kPfGather * 4);
      if (c.staged) {
        for (int j = lane; j < p.kcap; j += 32) o[j] = j < n ? pf_ld16(st + (uint32_t)j * 2) : -1;
      } else {
        for (int j = n + lane; j < p.kcap; j += 32) o[j] = -1;
      }
    }
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tmem_fence_after_sync();
    tmem_dealloc(tbase, kPfTmemCols);
  }
}

}  // namespace al
