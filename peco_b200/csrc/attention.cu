// Cluster-block-sparse attention on sm_100a tensor cores.
//
// Replaces the reference's WMMA kernel (peco/kernels/sparse_attention.cu:55-190):
// O = softmax(Q K^T / sqrt(D), masked by map[group(i), group(j)]) V, rows
// with no allowed key -> 0.
//
// Three kernels:
//  * planner (several CTAs per head): clamped cluster prefixes, the work units,
//    the key-row -> key-block map, zeroed padding rows of the key blocks, and
//    per unit the list of selected key clusters as block ranges.  A unit is
//    up to 128 consecutive query rows made of up to four whole consecutive
//    query groups (a group larger than 128 rows gets units of its own); its
//    key list is the union of its groups' selections, each entry tagged with
//    the groups that selected it, so the masks are per (row group, key
//    column).  Packing groups shares the key blocks they have in common (the
//    text groups every video group attends, and neighbouring clusters'
//    selections) and fills the 128-row tensor-core tile;
//  * pack (drop-in path only): row-major K/V -> key blocks (internal.h).  The
//    fused path writes key blocks straight from its quantise/gather kernel;
//  * main kernel (persistent, one CTA per SM).  Per unit, the selected key
//    blocks are concatenated and cut into 128-key tiles (16 blocks); a run of
//    consecutive blocks is ONE bulk copy.  Per tile t:
//      S[t%2]  = Q K^T         tcgen05.mma, A = Q (smem), B = K blocks (smem)
//      P       = exp2(S*c - m) 8 softmax warps: a query row is shared by two
//                              warps, each owning 64 key columns with its own
//                              running max (lazy rescale: only when it grows by
//                              > 8 in log2 units) and sum; P overwrites its half
//                              of S[t%2] in TMEM as 16-bit pairs
//      O_h    += P_h V_h       tcgen05.mma, A = P half h (TMEM), B = the V blocks
//                              of that half (smem, MN-major); O_0 and O_1 are
//                              separate accumulators
//    The epilogue merges the halves, O = (O_0 2^(m_0-M) + O_1 2^(m_1-M)) / L,
//    and can scatter rows through an inverse permutation (fusing
//    peco/clustering.py:127-136 into the output store).
// The MMA issuer runs one tile ahead (QK of tile t+1 before PV of tile t), so
// the tensor core computes the next scores while the softmax warps work on the
// current ones.  K and V stream through a 5-slot ring (two and a half tiles
// in flight), and Q is double-buffered so the next unit's tile arrives while
// the current unit runs.
//
// Warp roles: warp 0 = producer (unit claims, bulk copies, tile masks), warp
// 1 = MMA issuer (one thread) and TMEM owner, warps 2-9 = softmax + epilogue.
// CTAs claim units from a work counter, every head's text groups first.
// Every wait is bounded (common.cuh); on expiry the CTA records kDevTimeout in
// the device status word and unwinds.
#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

constexpr int kBM = kUnitRows;   // query rows per unit
constexpr int kBN = 128;         // keys per tile
constexpr int kTileBlocks = kBN / kKeyBlockRows;
constexpr int kSlots = 5;        // K/V ring: slot of K(t) = 2t mod 5, V(t) = 2t+1 mod 5
constexpr int kQBufs = 2;        // Q tiles: the next unit's loads while this one runs
constexpr int kRing = 8;         // tile-info ring depth
constexpr int kMaxGroups = 4;    // query groups per unit
constexpr int kPlanParts = 4;    // planner CTAs per head (at least)
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = 32 * (2 + kSoftmaxWarps);
constexpr uint32_t kTmemCols = 512;  // S0 | S1 | O_0 | O_1, 128 columns each

// tile-info flags
constexpr uint32_t kFirst = 1u, kLast = 2u, kEmpty = 4u, kEnd = 8u;

struct AttnArgs {
  const int* ws;              // plan workspace
  const unsigned char* kb;    // key blocks
  const unsigned char* vb;    // value blocks
  void* out;                  // [BH, out_rows, D]
  const int32_t* perm;        // optional [BH, video] inverse permutation for packed rows < video
  PlanGeom g;
  int bh;
  int out_rows;               // rows per head of the output tensor
  int video;                  // packed rows below this index go through perm
  float scale_log2;           // log2(e) / sqrt(D)
  unsigned* status;
};

struct TileInfo {
  uint32_t mask[kMaxGroups][4];  // per row group: key columns of the tile it attends
  int unit;                   // virtual unit index (local * BH + head)
  uint32_t flags;
  int shift;                  // TMEM lanes below this hold no row of the unit
  uint32_t bounds;            // bytes 0-2: first row (within the unit) of groups 1-3, 0xff = none
};
// A split unit's piece, part and part count ride in the tile flags above bit 8
// (each below 8: kSplitPieces, kSplitParts <= 4).
__device__ __forceinline__ uint32_t split_flags(int word) {
  return static_cast<uint32_t>(((word >> 16) & 7) << 6 | ((word >> 8) & 7) << 3 | (word & 7)) << 8;
}
__device__ __forceinline__ int split_word(uint32_t flags) {
  const int f = static_cast<int>(flags >> 8);
  return ((f >> 6) & 7) << 16 | ((f >> 3) & 7) << 8 | (f & 7);
}

struct __align__(8) Shared {
  uint64_t q_full[kQBufs], q_empty[kQBufs];
  uint64_t slot_full[kSlots], slot_empty[kSlots];
  uint64_t s_full[2], s_free[2], p_full[2];
  uint64_t o_full;
  uint64_t xch_full[4], xch_back[4];   // epilogue hand-off between the two warps of a row quarter
  uint64_t info_full[kRing], info_empty[kRing];
  TileInfo info[kRing];
  float2 xch[kBM];
  uint32_t tmem_base;
  int abort_flag;
};

// Q: D/64 panels of 128 rows x 128 bytes (128-byte swizzle, 8-row groups 1 KB
// apart).  K/V slots: 16 key blocks of 8 * D * 2 bytes.
template <int D>
struct Layout {
  static constexpr int kTileBytes = kBN * D * 2;
  static constexpr int kBlockBytes = kKeyBlockRows * D * 2;
  static constexpr int kQPanel = kBM * 128;
  static constexpr int kQ0 = 0;
  static constexpr int kSlot0 = kQBufs * kTileBytes;
  static constexpr int kShared = kSlot0 + kSlots * kTileBytes;
  static constexpr int kSmem = 1024 + kShared + static_cast<int>(sizeof(Shared));
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA exceeds the sm_100a limit");
};

__device__ __forceinline__ int* work_counter(const AttnArgs& a) {
  return const_cast<int*>(a.ws) + static_cast<long long>(a.bh - 1) * a.g.stride + (a.g.stride - 1);
}

// ---------------------------------------------------------------------------
// planner
// ---------------------------------------------------------------------------
__device__ long long block_exclusive_scan(long long v, long long* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  long long incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  __syncthreads();
  if (lane == 31) tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const long long t = lane < nw ? tmp[lane] : 0;
    long long inc = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += u;
    }
    tmp[lane] = inc - t;
  }
  __syncthreads();
  return tmp[warp] + incl - v;
}

// Query groups -> units, by all threads of the block.  The groups are visited
// in descending order (position k visits group G-1-k); a unit packs
// consecutive whole groups while their rows fit in kBM and there are at most
// kMaxGroups of them (empty groups included, but a unit never starts with
// one); a group of more than kBM rows gets units of its own, one per kBM
// rows.  As a sequential scan this is a chain of dependent shared-memory
// steps per group (~180 cycles each on one thread); here every position
// computes the unit that would start there and the position of the next
// start, and pointer doubling marks the starts reached from the first one.
// Writes ugroup[u] = first group << 3 | groups and urows[u] = rows, or for a
// piece of a large group -1 - (piece | part << 16 | parts << 24), for u < cap;
// returns the unit count (which may exceed cap).  With split > 1 the pieces
// of the first large group visited (at most kSplitPieces of them) become
// `split` units each, one per key-range part; *n_split is then their piece
// count (else 0).  scratch: 4 (G + 1) ints.
__device__ int pack_units(const int* gcount, int G, int cap, int* ugroup, int* urows, int* scratch, int split,
                          int* n_split) {
  int* fvs = scratch;               // [G + 1] first non-empty position >= x (G: none)
  int* ja = fvs + (G + 1);          // [G + 1] next start, then its doublings
  int* jb = ja + (G + 1);
  int* on = jb + (G + 1);           // [G + 1] 1: position starts a unit
  __shared__ int tmpi[32];
  __shared__ long long tmpl[32];
  __shared__ int carry, first_big;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  auto size_at = [&](int k) { return gcount[G - 1 - k]; };
  if (tid == 0) {
    first_big = G;
    *n_split = 0;
  }
  __syncthreads();
  for (int k = tid; k < G; k += blockDim.x)
    if (size_at(k) > kBM) atomicMin(&first_big, k);
  // 1. fvs: suffix minimum of (non-empty ? x : G), chunks from the top
  if (tid == 0) carry = G;
  __syncthreads();
  for (int hi = G; hi > 0; hi -= blockDim.x) {
    const int x = hi - 1 - tid;  // descending across threads: the suffix is a prefix in tid
    int v = (x >= 0 && size_at(x) > 0) ? x : G;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v = min(v, u);
    }
    if (lane == 31) tmpi[warp] = v;
    __syncthreads();
    int c = carry;
    for (int w2 = 0; w2 < warp; ++w2) c = min(c, tmpi[w2]);
    v = min(v, c);
    if (x >= 0) fvs[x] = v;
    __syncthreads();
    if (tid == blockDim.x - 1) carry = v;
    __syncthreads();
  }
  // 2. per position: end of the unit that would start there, next start
  for (int k = tid; k <= G; k += blockDim.x) {
    int nx = G;
    if (k < G && size_at(k) > 0) {
      int end = k + 1;
      if (size_at(k) <= kBM) {
        int rows = 0, ng = 0;
        end = k;
        while (end < G && ng < kMaxGroups) {
          const int n = size_at(end);
          if (n > kBM || rows + n > kBM) break;
          rows += n;
          ++ng;
          ++end;
        }
      }
      nx = end < G ? fvs[end] : G;
    }
    if (k == G) fvs[G] = G;
    ja[k] = nx;
    on[k] = 0;
  }
  __syncthreads();
  if (tid == 0) on[fvs[0]] = 1;  // fvs[0] == G: no unit at all (on[G] is a sentinel)
  __syncthreads();
  // 3. doubling: after round r every start within 2^(r+1) steps of the first
  // is marked (marks made during a round only reach further starts sooner)
  for (int span = 1; span <= G; span <<= 1) {
    for (int k = tid; k <= G; k += blockDim.x) {
      const int j = ja[k];
      if (on[k] && j < G) on[j] = 1;
      jb[k] = ja[j];
    }
    __syncthreads();
    int* t = ja;
    ja = jb;
    jb = t;
  }
  // 4. unit numbers: exclusive prefix of the units each start emits
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int k0 = 0; k0 < G; k0 += blockDim.x) {
    const int k = k0 + tid;
    int cnt = 0, parts = 1;
    if (k < G && on[k]) {
      const int n = size_at(k);
      const int pieces = (n + kBM - 1) / kBM;
      if (n > kBM && split > 1 && k == first_big && pieces <= kSplitPieces) {
        parts = split;
        *n_split = pieces;
      }
      cnt = n > kBM ? pieces * parts : 1;
    }
    const int u0 = carry + static_cast<int>(block_exclusive_scan(cnt, tmpl));
    if (cnt > 0) {
      const int q = G - 1 - k, n = size_at(k);
      if (n > kBM) {
        for (int i = 0; i < cnt; ++i)
          if (u0 + i < cap) {
            ugroup[u0 + i] = (q << 3) | 1;
            urows[u0 + i] = parts > 1 ? -1 - ((i / parts) | (i % parts) << 16 | parts << 24) : -1 - i;
          }
      } else if (u0 < cap) {
        int rows = 0, ng = 0, end = k;
        while (end < G && ng < kMaxGroups) {
          const int m = size_at(end);
          if (m > kBM || rows + m > kBM) break;
          rows += m;
          ++ng;
          ++end;
        }
        ugroup[u0] = ((G - end) << 3) | ng;  // first group = the last one visited
        urows[u0] = rows;
      }
    }
    __syncthreads();
    if (tid == blockDim.x - 1) carry = u0 + cnt;
    __syncthreads();
  }
  return carry;
}

// Group extents are clamped the way the reference's work map clamps them
// (sparse_attention.cu:25-31): start_g = min(S, sum_{g'<g} max(0, size_g')).
// Units of later query groups come first, so the text groups (which attend to
// every key) start early.  Several CTAs share a head (grid (BH, parts), at
// least kPlanParts, more when there are few heads): each recomputes the
// head's prefixes and unit list (cheap) and takes its slice of the key-row
// map, the padding rows and the units' entry lists; part 0 writes the per-head
// records.  Dynamic smem: 2 (gk + 1) + 2 gq + 2 max_units + 4 (gq + 1) ints,
// then (when ``map_in_smem``) the head's gq x gk map bytes, staged once so the
// per-unit entry scans read shared rather than global memory.
__global__ void __launch_bounds__(1024) attn_plan_kernel(const uint8_t* __restrict__ map,
                                                         const int* __restrict__ q_sizes,
                                                         const int* __restrict__ k_sizes, int* __restrict__ ws,
                                                         const PlanGeom g, unsigned char* k_blocks,
                                                         unsigned char* v_blocks, int block_bytes, int map_in_smem,
                                                         int split) {
  extern __shared__ int plan_sm[];
  int* skp = plan_sm;
  int* sgp = skp + g.gk + 1;
  int* gstart = sgp + g.gk + 1;
  int* gcount = gstart + g.gq;
  int* ugroup = gcount + g.gq;             // per unit: first group << 3 | groups
  int* urows = ugroup + g.max_units;         // per unit: rows
  int* pack_scratch = urows + g.max_units;   // 4 (gq + 1) ints for pack_units
  uint8_t* smap = reinterpret_cast<uint8_t*>(pack_scratch + 4 * (g.gq + 1));
  __shared__ long long tmp[32];
  __shared__ long long carry[2];
  __shared__ int n_units;
  const int head = blockIdx.x, part = blockIdx.y, parts = gridDim.y;
  const int tid = threadIdx.x, last = blockDim.x - 1;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  int* w = ws + static_cast<long long>(head) * g.stride;
  const int* qs = q_sizes + static_cast<long long>(head) * g.gq;
  const int* ks = k_sizes + static_cast<long long>(head) * g.gk;
  if (tid == 0) {
    carry[0] = carry[1] = 0;
    skp[0] = 0;
    sgp[0] = 0;
    if (head == gridDim.x - 1 && part == 0) w[g.stride - 1] = 0;  // work counter
  }
  __syncthreads();
  // key clusters: clamped row prefix and block prefix
  for (int c0 = 0; c0 < g.gk; c0 += blockDim.x) {
    const int c = c0 + tid;
    const long long v = c < g.gk ? max(0, ks[c]) : 0;
    const long long pre = carry[0] + block_exclusive_scan(v, tmp);
    const long long s0 = min(static_cast<long long>(g.sk), pre), s1 = min(static_cast<long long>(g.sk), pre + v);
    const long long nb = (s1 - s0 + kKeyBlockRows - 1) / kKeyBlockRows;
    const long long bpre = carry[1] + block_exclusive_scan(nb, tmp);
    if (c < g.gk) {
      skp[c + 1] = static_cast<int>(s1);
      sgp[c + 1] = static_cast<int>(bpre + nb);
    }
    __syncthreads();
    if (tid == last) {
      carry[0] = pre + v;
      carry[1] = bpre + nb;
    }
    __syncthreads();
  }
  if (part == 0)
    for (int c = tid; c <= g.gk; c += blockDim.x) {
      w[g.off_kp + c] = skp[c];
      w[g.off_gp + c] = sgp[c];
    }
  // query groups -> units
  if (tid == 0) carry[0] = 0;
  __syncthreads();
  for (int g0 = 0; g0 < g.gq; g0 += blockDim.x) {
    const int q = g0 + tid;
    const long long v = q < g.gq ? max(0, qs[q]) : 0;
    const long long pre = carry[0] + block_exclusive_scan(v, tmp);
    if (q < g.gq) {
      const long long s0 = min(static_cast<long long>(g.sq), pre), s1 = min(static_cast<long long>(g.sq), pre + v);
      gstart[q] = static_cast<int>(s0);
      gcount[q] = static_cast<int>(s1 - s0);
    }
    __syncthreads();
    if (tid == last) carry[0] = pre + v;
    __syncthreads();
  }
  int* units = w + g.off_units;
  // Units, later groups first (so the text groups, which attend every key,
  // start early): consecutive whole groups are packed while the rows fit in
  // kBM and there are at most kMaxGroups of them (a run of groups [lo, lo +
  // ng), empty ones included); a group larger than kBM rows gets units alone.
  {
    const int cap = static_cast<int>(g.max_units);
    __shared__ int n_split;
    const int nu = pack_units(gcount, g.gq, cap, ugroup, urows, pack_scratch, split, &n_split);
    if (tid == 0) {
      n_units = min(nu, cap);
      if (part == 0) {
        w[0] = n_units;
        w[1] = n_split;
      }
    }
    __syncthreads();
  }
  if (part == 0)
    for (int u = tid; u < n_units; u += blockDim.x) {
      const int lo = ugroup[u] >> 3, ng = ugroup[u] & 7;
      int* rec = units + kUnitInts * u;
      rec[7] = 0;
      if (urows[u] < 0) {  // piece of a large group (a key-range part of it when split)
        const int idx = -1 - urows[u];
        const int i = idx & 0xffff, prt = (idx >> 16) & 0xff, parts = idx >> 24;
        rec[0] = gstart[lo] + i * kBM;
        rec[1] = min(kBM, gcount[lo] - i * kBM);
        if (parts > 1) {
          rec[7] = (i << 16) | (prt << 8) | parts;
          if (prt == 0) {
            w[g.off_ptab + 2 * i] = rec[0];
            w[g.off_ptab + 2 * i + 1] = rec[1];
          }
        }
      } else {
        rec[0] = gstart[lo];
        rec[1] = urows[u];
      }
      unsigned bounds = 0xffffffu;  // bytes 0-2: first row of groups 1-3 within the unit
      for (int m = 1; m < ng; ++m)
        bounds = (bounds & ~(0xffu << (8 * (m - 1)))) | (static_cast<unsigned>(gstart[lo + m] - gstart[lo]) << (8 * (m - 1)));
      rec[4] = lo;
      rec[5] = ng;
      rec[6] = static_cast<int>(bounds);
    }
  // key row -> row of the key-block image
  int* rows = w + g.off_rows;
  for (int j = part * blockDim.x + tid; j < g.sk; j += parts * blockDim.x) {
    int lo = 0, hi = g.gk;  // largest c in [0, gk] with skp[c] <= j
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (skp[mid] <= j) lo = mid;
      else hi = mid - 1;
    }
    rows[j] = lo < g.gk ? kKeyBlockRows * sgp[lo] + (j - skp[lo]) : -1;
  }
  // zero the padding rows of every cluster's last block: eight lanes per
  // 128-byte row, so each warp store writes whole rows
  if (k_blocks) {
    const int panels = block_bytes / 1024;
    const int e = tid & 7;
    const long long n = static_cast<long long>(g.gk) * kKeyBlockRows * panels;
    for (long long idx = (part * blockDim.x + tid) >> 3; idx < n; idx += (parts * blockDim.x) >> 3) {
      const int p = static_cast<int>(idx % panels);
      const int ci = static_cast<int>(idx / panels);
      const int c = ci / kKeyBlockRows, i = ci % kKeyBlockRows;
      const int r = (skp[c + 1] - skp[c]) % kKeyBlockRows;
      if (r == 0 || i < r) continue;
      const long long off = (static_cast<long long>(head) * g.blocks + sgp[c + 1] - 1) * block_bytes + p * 1024 + i * 128;
      reinterpret_cast<uint4*>(k_blocks + off)[e] = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(v_blocks + off)[e] = make_uint4(0, 0, 0, 0);
    }
  }
  __syncthreads();
  const uint8_t* head_map = map + static_cast<long long>(head) * g.gq * g.gk;
  if (map_in_smem) {
    // eight independent loads in flight per thread, four map bytes per load
    // when the head's map is word-aligned (the shared copy always is)
    const int n = g.gq * g.gk;
    if ((reinterpret_cast<uintptr_t>(head_map) & 3) == 0) {
      const int nw = n >> 2;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(head_map);
      uint32_t* dst = reinterpret_cast<uint32_t*>(smap);
      for (int i0 = tid; i0 < nw; i0 += 8 * blockDim.x) {
        uint32_t b[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) b[e] = i0 + e * blockDim.x < nw ? src[i0 + e * blockDim.x] : 0u;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (i0 + e * blockDim.x < nw) dst[i0 + e * blockDim.x] = b[e];
      }
      for (int i = (nw << 2) + tid; i < n; i += blockDim.x) smap[i] = head_map[i];
    } else {
      for (int i0 = tid; i0 < n; i0 += 8 * blockDim.x) {
        uint8_t b[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) b[e] = i0 + e * blockDim.x < n ? head_map[i0 + e * blockDim.x] : 0;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (i0 + e * blockDim.x < n) smap[i0 + e * blockDim.x] = b[e];
      }
    }
    __syncthreads();
    head_map = smap;
  }
  // per unit: the selected key clusters as entries over the unit's block list
  int2* ent_all = reinterpret_cast<int2*>(w + g.off_ent);
  // units dealt round-robin over the head's CTAs first, so each CTA (and
  // scheduler) scans few of them
  for (int u = part + parts * warp; u < n_units; u += parts * nwarps) {
    const int lo = ugroup[u] >> 3, ng = ugroup[u] & 7;
    const uint8_t* mrow = head_map + static_cast<long long>(lo) * g.gk;
    int2* ent = ent_all + static_cast<long long>(u) * g.gk;
    int nent = 0, blocks = 0;
    // the map bytes of kMapBatch chunks of 32 clusters are loaded together,
    // so one memory round trip serves kMapBatch * 32 clusters
    constexpr int kMapBatch = 8;
    int gms[kMapBatch];
    for (int c0 = 0; c0 < g.gk; c0 += 32) {
      const int c = c0 + lane;
      const int bi = (c0 / 32) % kMapBatch;
      if (bi == 0) {
#pragma unroll
        for (int b = 0; b < kMapBatch; ++b) {
          const int cb = c + 32 * b;
          int v = 0;
          if (cb < g.gk)
            for (int m = 0; m < ng; ++m) v |= (mrow[static_cast<long long>(m) * g.gk + cb] ? 1 : 0) << m;
          gms[b] = v;
        }
      }
      int gm = 0;
#pragma unroll
      for (int b = 0; b < kMapBatch; ++b) gm = b == bi ? gms[b] : gm;
      int n = 0, nb = 0;
      if (c < g.gk) {
        n = skp[c + 1] - skp[c];
        if (n > 0 && gm) nb = sgp[c + 1] - sgp[c];
      }
      const unsigned bal = __ballot_sync(0xffffffffu, nb > 0);
      int incl = nb;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (nb > 0) {
        const int pe = blocks + incl;
        const int idx = nent + __popc(bal & ((1u << lane) - 1u));
        // (end position, groups that selected the cluster, rows in its last block)
        ent[idx] = make_int2(sgp[c] - (pe - nb), (pe << 8) | (gm << 4) | (n - kKeyBlockRows * (nb - 1)));
      }
      nent += __popc(bal);
      blocks += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      units[kUnitInts * u + 2] = nent;
      units[kUnitInts * u + 3] = blocks;
    }
  }
}

// row-major K/V [BH, SK, D] -> key blocks (rows without a block are skipped)
template <int D>
__global__ void pack_key_blocks_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v,
                                       unsigned char* __restrict__ kb, unsigned char* __restrict__ vb,
                                       const int* __restrict__ ws, const PlanGeom g, int bh, unsigned* status) {
  constexpr int kChunks = D / 8;
  const long long total = static_cast<long long>(bh) * g.sk * kChunks;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int chunk = static_cast<int>(idx % kChunks);
    const long long row = idx / kChunks;
    const int head = static_cast<int>(row / g.sk);
    const int j = static_cast<int>(row - static_cast<long long>(head) * g.sk);
    const int dst = ws[static_cast<long long>(head) * g.stride + g.off_rows + j];
    if (dst < 0) continue;
    if (dst >= g.blocks * kKeyBlockRows) {
      if (chunk == 0) record_status(status, kDevBadIndex);
      continue;
    }
    const long long off = (static_cast<long long>(head) * g.blocks + dst / kKeyBlockRows) * (kKeyBlockRows * D * 2) +
                          key_block_offset(dst % kKeyBlockRows, chunk * 8);
    *reinterpret_cast<uint4*>(kb + off) = k[idx];
    *reinterpret_cast<uint4*>(vb + off) = v[idx];
  }
}

// ---------------------------------------------------------------------------
// main kernel (persistent)
// ---------------------------------------------------------------------------
template <int D, int AB, bool SPLIT>  // AB: 0 = fp16, 1 = bf16; SPLIT: the plan may hold split key ranges
__global__ void __launch_bounds__(kThreads, 1) sparse_attention_tc(const __grid_constant__ CUtensorMap qmap,
                                                                  const AttnArgs args) {
  using L = Layout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1 KB-aligned base, derived from smem_raw by pointer arithmetic so that
  // the compiler keeps shared-memory (not generic) accesses through it
  unsigned char* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Shared& sh = *reinterpret_cast<Shared*>(base + L::kShared);
  volatile int* abort_flag = &sh.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const PlanGeom& g = args.g;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQBufs; ++i) {
      mbar_init(&sh.q_full[i], 1);
      mbar_init(&sh.q_empty[i], 1);
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sh.slot_full[i], 1);
      mbar_init(&sh.slot_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.s_full[i], 1);
      mbar_init(&sh.s_free[i], 1);
      mbar_init(&sh.p_full[i], kSoftmaxWarps);
    }
    mbar_init(&sh.o_full, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&sh.xch_full[i], 1);
      mbar_init(&sh.xch_back[i], 1);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&sh.info_full[i], 1);
      mbar_init(&sh.info_empty[i], 1 + kSoftmaxWarps);
    }
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  // blocks past a tile's end are never loaded: zero the ring once so the
  // tensor core only ever sees finite values there
  for (int i = threadIdx.x; i < kSlots * L::kTileBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(base + L::kSlot0)[i] = make_uint4(0, 0, 0, 0);
  fence_async_smem();
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------- producer
    if (lane == 0) prefetch_tensormap(&qmap);
    bool ok = true;
    int tile = 0;      // tiles issued by this CTA
    int entry = 0;     // info entries pushed
    int qloads = 0;    // Q tiles loaded
    // lane i < 16 writes mask word i (group i / 4, word i % 4)
    int unit_split = 0;  // split word of the unit being issued
    auto push_info = [&](uint32_t my_word, int unit, uint32_t flags, int shift, uint32_t bounds) {
      const int slot = entry % kRing;
      if (ok && entry >= kRing) ok = mbar_wait_warp(&sh.info_empty[slot], ((entry / kRing) - 1) & 1, abort_flag, args.status);
      if (ok) {
        TileInfo& ti = sh.info[slot];
        if (lane < 4 * kMaxGroups) ti.mask[lane >> 2][lane & 3] = my_word;
        if (lane == 0) {
          ti.unit = unit;
          ti.flags = SPLIT ? (flags | split_flags(unit_split)) : flags;
          ti.shift = shift;
          ti.bounds = bounds;
        }
      }
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&sh.info_full[slot]);
      __syncwarp();
      ++entry;
    };
    const long long total_units = static_cast<long long>(args.bh) * g.max_units;
    for (;;) {
      // ---- claim a unit
      int got = 0;
      if (lane == 0) got = atomicAdd(work_counter(args), 1);
      const int v = __shfl_sync(0xffffffffu, got, 0);  // unit indices fit in int (checked at launch)
      if (v >= total_units || !ok) break;
      const int head = v % args.bh;
      const int local = v / args.bh;
      const int* w = args.ws + static_cast<long long>(head) * g.stride;
      if (local >= w[0] || local >= g.max_units) continue;
      const int4 rec = *reinterpret_cast<const int4*>(w + g.off_units + kUnitInts * local);
      const int4 rec2 = *reinterpret_cast<const int4*>(w + g.off_units + kUnitInts * local + 4);
      const uint32_t bounds = static_cast<uint32_t>(rec2.z);
      const int q_start = rec.x;
      // the unit's rows fill the TOP lanes of the 128-row tile (lanes
      // shift..127): lane quarters 0 and 1, whose schedulers also run the
      // producer and MMA warps, are the ones left without rows
      const int shift = kBM - min(max(rec.y, 0), kBM);
      int nent = rec.z, nblk = rec.w;
      if (nent < 0 || nent > g.gk || nblk < 0) {  // not a plan of this geometry
        if (lane == 0) record_status(args.status, kDevBadIndex);
        nent = nblk = 0;
      }
      // a split unit walks only its part of the key tiles
      const int ntiles_all = (nblk + kTileBlocks - 1) / kTileBlocks;
      int t_begin = 0, t_end = ntiles_all;
      const int parts = SPLIT ? (rec2.w & 0xff) : 1, prt = SPLIT ? ((rec2.w >> 8) & 0xff) : 0;
      if (SPLIT) unit_split = rec2.w;
      if (SPLIT && parts > 1) {
        const int per = (ntiles_all + parts - 1) / parts;
        t_begin = min(ntiles_all, prt * per);
        t_end = min(ntiles_all, t_begin + per);
      }
      if (nblk == 0 || t_begin >= t_end) {
        push_info(0u, static_cast<int>(v), kEmpty, shift, bounds);  // no key at all: rows are zero
        if (!ok) break;
        continue;
      }
      const int2* ents = reinterpret_cast<const int2*>(w + g.off_ent) + static_cast<long long>(local) * g.gk;
      const long long block0 = static_cast<long long>(head) * g.blocks;
      // window of 32 entries, one per lane: block offset, end position, rows
      // in the last block, groups of the unit that attend the cluster
      int w0 = 0, wz = 0, wend = 0x7fffffff, wlast = 0, wgm = 0;
      auto load_window = [&](int from) {
        w0 = from;
        wz = 0;
        wend = 0x7fffffff;
        wlast = 0;
        wgm = 0;
        if (from + lane < nent) {
          const int2 e = ents[from + lane];
          wz = e.x;
          wend = e.y >> 8;
          wgm = (e.y >> 4) & 15;
          wlast = e.y & 15;
        }
      };
      load_window(0);
      // a later part: move the window up to its first tile's blocks
      for (; SPLIT;) {
        const int passed = __popc(__ballot_sync(0xffffffffu, wend <= t_begin * kTileBlocks));
        if (passed > 32 - kTileBlocks && w0 + 32 < nent) load_window(w0 + passed);
        else break;
      }
      for (int t = t_begin; t < t_end && ok; ++t) {
        const int p0 = t * kTileBlocks;
        const int before = __popc(__ballot_sync(0xffffffffu, wend <= p0));
        if (before > 32 - kTileBlocks && w0 + 32 < nent) load_window(w0 + before);
        // lane < ngroups: block of tile position lane (binary search over the window)
        const int pos = p0 + lane;
        int k = 0;
#pragma unroll
        for (int step = 16; step >= 1; step >>= 1) {
          const int e = __shfl_sync(0xffffffffu, wend, k + step - 1);
          if (e <= pos) k += step;
        }
        const int kz = __shfl_sync(0xffffffffu, wz, k);
        const int kend = __shfl_sync(0xffffffffu, wend, k);
        const int klast = __shfl_sync(0xffffffffu, wlast, k);
        const int kgm = __shfl_sync(0xffffffffu, wgm, k);
        const int ngroups = min(kTileBlocks, nblk - p0);
        int blk = 0, valid = 0;
        if (lane < ngroups) {
          blk = kz + pos;
          valid = pos == kend - 1 ? klast : kKeyBlockRows;
        }
        // ---- K and V of the tile: one bulk copy per run of consecutive blocks
        const int kitem = 2 * tile, vitem = kitem + 1;
        const int ks = kitem % kSlots, vs = vitem % kSlots;
        if (ok && kitem >= kSlots) ok = mbar_wait_warp(&sh.slot_empty[ks], ((kitem / kSlots) - 1) & 1, abort_flag, args.status);
        if (ok && vitem >= kSlots) ok = mbar_wait_warp(&sh.slot_empty[vs], ((vitem / kSlots) - 1) & 1, abort_flag, args.status);
        if (!ok) break;
        if (lane == 0) {
          const uint32_t bytes = static_cast<uint32_t>(ngroups) * L::kBlockBytes;
          mbar_arrive_expect_tx(&sh.slot_full[ks], bytes);
          mbar_arrive_expect_tx(&sh.slot_full[vs], bytes);
        }
        __syncwarp();
        const int prev = __shfl_up_sync(0xffffffffu, blk, 1);
        const bool cont = lane > 0 && lane < ngroups && blk == prev + 1;
        const unsigned cmask = __ballot_sync(0xffffffffu, cont);
        int n = 0;  // blocks of the run this lane starts (0 if none)
        // the run ends at the first non-continuation lane above this one
        // (lanes >= ngroups never continue, and ngroups <= 16 keeps the shift < 32)
        if (lane < ngroups && !cont) n = __ffs(~cmask & (0xffffffffu << (lane + 1))) - 1 - lane;
        // lanes 0-15 copy K, lanes 16-31 copy V of the run that lane - 16 starts
        const int src = lane & (kTileBlocks - 1);
        const int rn = __shfl_sync(0xffffffffu, n, src);
        const int rb = __shfl_sync(0xffffffffu, blk, src);
        if (rn > 0 && (rb < 0 || rb + rn > g.blocks)) {
          // a block outside this head: skip the copy (the tile's wait then
          // expires and the call reports the error)
          record_status(args.status, kDevBadIndex);
        } else if (rn > 0) {
          const bool is_v = lane >= kTileBlocks;
          const int sl = is_v ? vs : ks;
          const unsigned char* gsrc = (is_v ? args.vb : args.kb) + (block0 + rb) * L::kBlockBytes;
          bulk_load(base + L::kSlot0 + sl * L::kTileBytes + src * L::kBlockBytes, gsrc,
                    static_cast<uint32_t>(rn) * L::kBlockBytes, &sh.slot_full[sl]);
        }
        __syncwarp();
        if (t == t_begin) {
          // first tile of the unit: its Q tile, once the previous unit's last
          // QK has released the buffer (its K/V are already in flight)
          const int qb = qloads % kQBufs, qu = qloads / kQBufs;
          if (ok && qu > 0) ok = mbar_wait_warp(&sh.q_empty[qb], (qu - 1) & 1, abort_flag, args.status);
          if (lane == 0 && ok) {
            mbar_arrive_expect_tx(&sh.q_full[qb], L::kTileBytes);
#pragma unroll
            for (int p = 0; p < D / 64; ++p)
              tma_load_2d(base + L::kQ0 + qb * L::kTileBytes + p * L::kQPanel, &qmap, 64 * p,
                          static_cast<int>(static_cast<long long>(head) * g.sq + q_start - shift), &sh.q_full[qb]);
          }
          __syncwarp();
          ++qloads;
        }
        // per block (lane): valid rows, one byte per group that attends it;
        // lane i < 16 then assembles mask word i % 4 of group i / 4 (the
        // bytes of blocks 4 (i % 4) .. 4 (i % 4) + 3)
        const unsigned bits = lane < ngroups ? ((1u << valid) - 1u) : 0u;
        unsigned bytes = 0;
#pragma unroll
        for (int m = 0; m < kMaxGroups; ++m) bytes |= ((kgm >> m) & 1) ? bits << (8 * m) : 0u;
        const int wi = lane & 3, gi = (lane >> 2) & 3;
        uint32_t my_word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const unsigned bb = __shfl_sync(0xffffffffu, bytes, 4 * wi + e);
          my_word |= ((bb >> (8 * gi)) & 0xffu) << (8 * e);
        }
        push_info(my_word, static_cast<int>(v), (t == t_begin ? kFirst : 0u) | (t == t_end - 1 ? kLast : 0u), shift,
                  bounds);
        ++tile;
        if (*abort_flag) ok = false;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
      if (!ok) break;
    }
    push_info(0u, -1, kEnd, 0, 0xffffffu);
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t idesc_qk = instr_desc(128, kBN, AB, false, false);
      constexpr uint32_t idesc_pv = instr_desc(128, D, AB, false, true);
      bool ok = true;
      int entry = 0, t = 0, qloads = 0, qbuf = 0;
      int cur = -1;  // tile whose P.V is pending
      uint32_t cur_flags = 0;
      auto issue_pv = [&]() {
        const int b = cur & 1, item = 2 * cur + 1, sl = item % kSlots;
        ok = mbar_wait(&sh.p_full[b], (cur >> 1) & 1, abort_flag, args.status);
        if (ok) ok = mbar_wait(&sh.slot_full[sl], (item / kSlots) & 1, abort_flag, args.status);
        if (!ok) return;
        tc_fence_after();
        const uint32_t va = smem_u32(base + L::kSlot0 + sl * L::kTileBytes);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int kk = 0; kk < kBN / 32; ++kk) {
            // 16 keys = two blocks; MN-major V: 64-dim panels 1 KB apart, 8-key groups one block apart
            const uint64_t bdesc = smem_desc(va + (8 * h + 2 * kk) * L::kBlockBytes, 1024, L::kBlockBytes);
            umma_ts(tmem + 256 + 128 * h, tmem + b * 128 + 64 * h + kk * 8, bdesc, idesc_pv,
                    ((cur_flags & kFirst) && kk == 0) ? 0u : 1u);
          }
        }
        umma_commit(&sh.s_free[b]);
        umma_commit(&sh.slot_empty[sl]);
        if (cur_flags & kLast) umma_commit(&sh.o_full);
      };
      for (;;) {
        const int slot = entry % kRing;
        ok = mbar_wait(&sh.info_full[slot], (entry / kRing) & 1, abort_flag, args.status);
        if (!ok) break;
        const uint32_t fl = sh.info[slot].flags;
        mbar_arrive(&sh.info_empty[slot]);
        ++entry;
        if (fl & kEnd) break;
        if (fl & kEmpty) continue;
        // ---- S[t%2] = Q K^T for the next tile
        const int b = t & 1, item = 2 * t, sl = item % kSlots;
        if (fl & kFirst) {
          qbuf = qloads % kQBufs;
          ok = mbar_wait(&sh.q_full[qbuf], (qloads / kQBufs) & 1, abort_flag, args.status);
          ++qloads;
        }
        if (ok) ok = mbar_wait(&sh.slot_full[sl], (item / kSlots) & 1, abort_flag, args.status);
        if (ok && t >= 2) ok = mbar_wait(&sh.s_free[b], ((t >> 1) - 1) & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(base + L::kQ0 + qbuf * L::kTileBytes);
        const uint32_t ka = smem_u32(base + L::kSlot0 + sl * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t col = (kk & 3) * 32;
          umma_ss(tmem + b * 128, smem_desc(qa + (kk >> 2) * L::kQPanel + col, 16, 1024),
                  smem_desc(ka + (kk >> 2) * 1024 + col, 16, L::kBlockBytes), idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sh.s_full[b]);
        umma_commit(&sh.slot_empty[sl]);
        if (fl & kLast) umma_commit(&sh.q_empty[qbuf]);
        // ---- O += P V for the previous tile
        if (cur >= 0) {
          issue_pv();
          if (!ok) break;
        }
        cur = t;
        cur_flags = fl;
        ++t;
      }
      if (ok && cur >= 0) issue_pv();
      // drain our MMAs before TMEM is released
      if (cur >= 0) mbar_wait(&sh.s_free[cur & 1], (cur >> 1) & 1, abort_flag, args.status);
    }
    __syncwarp();
  } else {
    // ----------------------------------------------- softmax + epilogue
    using T = typename std::conditional<AB == 1, __nv_bfloat16, __half>::type;
    const int quarter = warp & 3;                  // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;              // key columns [64 half, 64 half + 64)
    const int r = quarter * 32 + lane;             // query row within the unit
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_own = tmem + 256 + 128 * half;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    int entry = 0, t = 0, units_done = 0;
    // output row of unit v for this thread (nullptr: not a real row)
    auto out_row = [&](int v) -> T* {
      const int head = v % args.bh, local = v / args.bh;
      const int* rec = args.ws + static_cast<long long>(head) * g.stride + g.off_units + kUnitInts * local;
      const int q_start = rec[0], q_count = min(max(rec[1], 0), kBM);
      const int rr = r - (kBM - q_count);  // rows fill the top lanes
      if (rr < 0) return nullptr;
      const int prow = q_start + rr;
      long long orow = prow;
      if (args.perm && prow < args.video) orow = args.perm[static_cast<long long>(head) * args.video + prow];
      if (orow < 0 || orow >= args.out_rows) {
        record_status(args.status, kDevBadIndex);
        return nullptr;
      }
      return static_cast<T*>(args.out) + (static_cast<long long>(head) * args.out_rows + orow) * D + (D / 2) * half;
    };
    // a split unit's partial results for this thread's row: O (fp32,
    // unnormalised, kPartCols columns) and (max, sum) in the workspace;
    // split = 0 for a whole unit
    auto part_row = [&](int v, int sp, int row_shift, int& split, float*& ml) -> float* {
      const int head = v % args.bh;
      const int* wh = args.ws + static_cast<long long>(head) * g.stride;
      split = (sp & 0xff) > 1 ? 1 : 0;
      ml = nullptr;
      if (!split) return nullptr;
      const int rr = r - row_shift;
      const int piece = sp >> 16, prt = (sp >> 8) & 0xff;
      if (rr < 0 || piece >= kSplitPieces || prt >= kSplitParts) return nullptr;
      const long long row = static_cast<long long>(piece * kSplitParts + prt) * kUnitRows + rr;
      float* wf = reinterpret_cast<float*>(const_cast<int*>(wh));
      ml = wf + g.off_ml + 2 * row;
      return wf + g.off_part + row * kPartCols;
    };
    for (;;) {
      const int slot = entry % kRing;
      ok = mbar_wait_warp(&sh.info_full[slot], (entry / kRing) & 1, abort_flag, args.status);
      if (!ok) break;
      // read what this thread needs before the slot is released: the tile's
      // flags and unit, and the two mask words of this row's group
      const TileInfo& ts = sh.info[slot];
      TileInfo ti;
      ti.flags = ts.flags;
      ti.unit = ts.unit;
      ti.shift = ts.shift;
      const uint32_t tb = ts.bounds;
      const int rr = r - ti.shift;
      const int grp = (rr >= static_cast<int>(tb & 0xffu)) + (rr >= static_cast<int>((tb >> 8) & 0xffu)) +
                      (rr >= static_cast<int>((tb >> 16) & 0xffu));
      const uint32_t mw[2] = {ts.mask[grp][2 * half], ts.mask[grp][2 * half + 1]};
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.info_empty[slot]);
      ++entry;
      if (ti.flags & kEnd) break;
      if (ti.flags & kEmpty) {
        int split;
        float* ml;
        split = 0;
        if (SPLIT) part_row(ti.unit, split_word(ti.flags), ti.shift, split, ml);
        if (SPLIT && split) {  // a key-range part with no tile: contributes nothing
          if (half == 0 && ml) {
            ml[0] = -INFINITY;
            ml[1] = 0.0f;
          }
        } else {
          T* dst = out_row(ti.unit);
          if (dst) {
#pragma unroll
            for (int c = 0; c < D / 16; ++c) reinterpret_cast<uint4*>(dst)[c] = make_uint4(0, 0, 0, 0);
          }
        }
        __syncwarp();
        continue;
      }
      if (ti.flags & kFirst) {
        m = -INFINITY;
        l = 0.0f;
      }
      const int b = t & 1;
      ok = mbar_wait_warp(&sh.s_full[b], (t >> 1) & 1, abort_flag, args.status);
      if (!ok) break;
      // a warp whose 32 lanes hold no row of the unit skips the softmax: the
      // P.V of its lanes then reads stale TMEM, which only feeds O rows that
      // are never stored
      const bool idle = quarter * 32 + 31 < ti.shift;
      if (!idle) {
      tc_fence_after();
      constexpr int kCols = kBN / 2;
      float s[kCols];
#pragma unroll
      for (int c = 0; c < kCols / 32; ++c) {
        uint32_t vv[32];
        tmem_ld32_sync(tmem + b * 128 + 64 * half + lane_off + c * 32, vv);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[c * 32 + j] = __uint_as_float(vv[j]);
      }
      // raw scores of masked keys become -inf; the row max runs in kChains
      // independent chains over column pairs (three-input max), and the
      // scale (> 0) commutes with it
      constexpr int kChains = 8;
      float mxc[kChains];
#pragma unroll
      for (int i = 0; i < kChains; ++i) mxc[i] = -INFINITY;
#pragma unroll
      for (int j = 0; j < kCols; j += 2) {
        const bool v0 = (mw[j >> 5] >> (j & 31)) & 1u;
        const bool v1 = (mw[j >> 5] >> ((j + 1) & 31)) & 1u;
        s[j] = v0 ? s[j] : -INFINITY;
        s[j + 1] = v1 ? s[j + 1] : -INFINITY;
        mxc[(j / 2) % kChains] = fmaxf(mxc[(j / 2) % kChains], fmaxf(s[j], s[j + 1]));
      }
#pragma unroll
      for (int i = kChains / 2; i > 0; i >>= 1) {
#pragma unroll
        for (int k2 = 0; k2 < i; ++k2) mxc[k2] = fmaxf(mxc[k2], mxc[k2 + i]);
      }
      const float mx = mxc[0] * args.scale_log2;
      // grow the running max lazily (only by > 8 in log2 units); rescaling O
      // is warp-collective (tcgen05.ld/st are .sync.aligned) and needs the
      // previous tile's P.V to be complete
      const bool grow = (mx > m + 8.0f) || (m == -INFINITY && mx > -INFINITY);
      const bool rescale_me = grow && m != -INFINITY;
      if (__any_sync(0xffffffffu, rescale_me)) {
        ok = mbar_wait_warp(&sh.s_free[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
        const float f = rescale_me ? exp2_approx(m - mx) : 1.0f;
        l *= f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t vv[32];
          tmem_ld32_sync(o_own + lane_off + c * 32, vv);
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            lo[j] = __float_as_uint(__uint_as_float(vv[j]) * f);
            hi[j] = __float_as_uint(__uint_as_float(vv[16 + j]) * f);
          }
          tmem_st16(o_own + lane_off + c * 32, lo);
          tmem_st16(o_own + lane_off + c * 32 + 16, hi);
        }
      }
      if (grow) m = mx;
      // p = 2^(s*c - m): one paired FFMA per two scores and one ex2 per score
      // (masked: 2^-inf = 0); the row sum runs in kChains / 2 paired chains
      const float neg_m = (m == -INFINITY) ? 0.0f : -m;
      const float2 c2 = make_float2(args.scale_log2, args.scale_log2), nm2 = make_float2(neg_m, neg_m);
      float2 sum2[kChains / 2];
#pragma unroll
      for (int i = 0; i < kChains / 2; ++i) sum2[i] = make_float2(0.0f, 0.0f);
      uint32_t packed[kCols / 2];
#pragma unroll
      for (int j = 0; j < kCols; j += 2) {
        const float2 a2 = ffma2(make_float2(s[j], s[j + 1]), c2, nm2);
        const float p0 = exp2_approx(a2.x), p1 = exp2_approx(a2.y);
        sum2[(j / 2) % (kChains / 2)] = fadd2(sum2[(j / 2) % (kChains / 2)], make_float2(p0, p1));
        packed[j >> 1] = AB ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
      }
#pragma unroll
      for (int i = kChains / 4; i > 0; i >>= 1) {
#pragma unroll
        for (int k2 = 0; k2 < i; ++k2) sum2[k2] = fadd2(sum2[k2], sum2[k2 + i]);
      }
      l += sum2[0].x + sum2[0].y;
#pragma unroll
      for (int c = 0; c < kCols / 32; ++c) {
        uint32_t part[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) part[j] = packed[c * 16 + j];
        tmem_st16(tmem + b * 128 + 64 * half + lane_off + c * 16, part);
      }
      tmem_st_wait();
      tc_fence_before();
      }  // !idle
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.p_full[b]);
      ++t;
      if (ti.flags & kLast) {
        // epilogue of the unit: O_0 and O_1 are final once its last P.V completes
        ok = mbar_wait_warp(&sh.o_full, units_done & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
        // merge factors: half 1 hands (m, l) to half 0, which returns the
        // scale of each accumulator with 1/L folded in (a split part keeps O
        // unnormalised and records its max and sum instead)
        int split = 0;
        float* ml = nullptr;
        float* prow = (!SPLIT || idle) ? nullptr : part_row(ti.unit, split_word(ti.flags), ti.shift, split, ml);
        float a0, a1;
        if (half == 1) {
          sh.xch[r] = make_float2(m, l);
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.xch_full[quarter]);
          ok = mbar_wait_warp(&sh.xch_back[quarter], units_done & 1, abort_flag, args.status);
          if (!ok) break;
          const float2 f = sh.xch[r];
          a0 = f.x;
          a1 = f.y;
        } else {
          ok = mbar_wait_warp(&sh.xch_full[quarter], units_done & 1, abort_flag, args.status);
          if (!ok) break;
          const float2 o = sh.xch[r];
          const float mm = fmaxf(m, o.x);
          const float e0 = m == -INFINITY ? 0.0f : exp2_approx(m - mm);
          const float e1 = o.x == -INFINITY ? 0.0f : exp2_approx(o.x - mm);
          const float tot = l * e0 + o.y * e1;
          const float inv = tot > 0.0f ? 1.0f / tot : 0.0f;
          a0 = (SPLIT && split) ? e0 : e0 * inv;
          a1 = (SPLIT && split) ? e1 : e1 * inv;
          if (SPLIT && split && ml) {
            ml[0] = mm;
            ml[1] = tot;
          }
          sh.xch[r] = make_float2(a0, a1);
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.xch_back[quarter]);
        }
        ++units_done;
        T* dst = (idle || (SPLIT && split)) ? nullptr : out_row(ti.unit);
        __syncwarp();
#pragma unroll
        for (int c = 0; c < D / 64 && !idle; ++c) {
          // this warp writes output dims [D/2 half, D/2 (half + 1))
          uint32_t v0[32], v1[32];
          tmem_ld32_sync(tmem + 256 + lane_off + (D / 2) * half + c * 32, v0);
          tmem_ld32_sync(tmem + 384 + lane_off + (D / 2) * half + c * 32, v1);
          if (SPLIT && split && prow) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              float4 f;
              f.x = __uint_as_float(v0[j]) * a0 + __uint_as_float(v1[j]) * a1;
              f.y = __uint_as_float(v0[j + 1]) * a0 + __uint_as_float(v1[j + 1]) * a1;
              f.z = __uint_as_float(v0[j + 2]) * a0 + __uint_as_float(v1[j + 2]) * a1;
              f.w = __uint_as_float(v0[j + 3]) * a0 + __uint_as_float(v1[j + 3]) * a1;
              reinterpret_cast<float4*>(prow + (D / 2) * half + c * 32)[j / 4] = f;
            }
          }
          if (dst) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 pk;
              uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float x0 = __uint_as_float(v0[j + 2 * e]) * a0 + __uint_as_float(v1[j + 2 * e]) * a1;
                const float x1 = __uint_as_float(v0[j + 2 * e + 1]) * a0 + __uint_as_float(v1[j + 2 * e + 1]) * a1;
                pw[e] = AB ? pack_bf16x2(x0, x1) : pack_f16x2(x0, x1);
              }
              reinterpret_cast<uint4*>(dst)[(c * 32 + j) / 8] = pk;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

bool make_rows_map(CUtensorMap* m, const void* base, long long rows, int dims, int box_rows, int dtype) {
  const uint64_t gdims[2] = {static_cast<uint64_t>(dims), static_cast<uint64_t>(rows)};
  const uint64_t gstr[1] = {static_cast<uint64_t>(dims) * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(box_rows)};
  return encode_tensor_map(m, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                           base, gdims, gstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return kNumSMs;
  return n > 0 ? n : kNumSMs;
}

// Merge the key-range parts of every split piece: per row, max M = max_p M_p,
// sum L = sum_p L_p 2^(M_p - M), O = sum_p O_p 2^(M_p - M) / L (a row no part
// attended stays zero), written through the same output mapping as the main
// kernel's epilogue.  Grid (kSplitPieces, BH, D / 8): one thread per (row,
// 8 output columns), so every thread's loads are in flight together.
template <int D, int AB>
__global__ void __launch_bounds__(kUnitRows) split_combine_kernel(const AttnArgs a) {
  using T = typename std::conditional<AB == 1, __nv_bfloat16, __half>::type;
  const PlanGeom& g = a.g;
  const int piece = blockIdx.x, head = blockIdx.y, rr = threadIdx.x, c = 8 * static_cast<int>(blockIdx.z);
  const int* wh = a.ws + static_cast<long long>(head) * g.stride;
  if (piece >= min(wh[1], kSplitPieces)) return;
  const int q_start = wh[g.off_ptab + 2 * piece], q_count = min(max(wh[g.off_ptab + 2 * piece + 1], 0), kUnitRows);
  if (rr >= q_count) return;
  const float* wf = reinterpret_cast<const float*>(wh);
  float mp[kSplitParts], lp[kSplitParts];
  float mx = -INFINITY;
#pragma unroll
  for (int p = 0; p < kSplitParts; ++p) {
    const long long row = static_cast<long long>(piece * kSplitParts + p) * kUnitRows + rr;
    mp[p] = wf[g.off_ml + 2 * row];
    lp[p] = wf[g.off_ml + 2 * row + 1];
    mx = fmaxf(mx, mp[p]);
  }
  float wgt[kSplitParts];
  float tot = 0.0f;
#pragma unroll
  for (int p = 0; p < kSplitParts; ++p) {
    wgt[p] = (mx == -INFINITY || mp[p] == -INFINITY) ? 0.0f : exp2f(mp[p] - mx);
    tot += lp[p] * wgt[p];
  }
  const float inv = tot > 0.0f ? 1.0f / tot : 0.0f;
  const int prow = q_start + rr;
  long long orow = prow;
  if (a.perm && prow < a.video) orow = a.perm[static_cast<long long>(head) * a.video + prow];
  if (orow < 0 || orow >= a.out_rows) {
    record_status(a.status, kDevBadIndex);
    return;
  }
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll
  for (int p = 0; p < kSplitParts; ++p) {
    if (wgt[p] == 0.0f) continue;
    const float* src = wf + g.off_part + (static_cast<long long>(piece * kSplitParts + p) * kUnitRows + rr) * kPartCols + c;
    const float4 x0 = reinterpret_cast<const float4*>(src)[0], x1 = reinterpret_cast<const float4*>(src)[1];
    const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += xs[e] * wgt[p];
  }
  uint4 pk;
  uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
  for (int e = 0; e < 4; ++e)
    pw[e] = AB ? pack_bf16x2(acc[2 * e] * inv, acc[2 * e + 1] * inv) : pack_f16x2(acc[2 * e] * inv, acc[2 * e + 1] * inv);
  T* dst = static_cast<T*>(a.out) + (static_cast<long long>(head) * a.out_rows + orow) * D;
  reinterpret_cast<uint4*>(dst)[c / 8] = pk;
}

template <int D, int AB>
int launch_main(const void* q, const AttnArgs& a, cudaStream_t stream) {
  CUtensorMap qmap;
  if (!make_rows_map(&qmap, q, static_cast<long long>(a.bh) * a.g.sq, D, kBM, AB)) return kErrTensorMap;
  const int smem = Layout<D>::kSmem;
  const bool split = attention_split_parts(a.bh, a.g.sk) > 1;
  cudaError_t e = split ? cudaFuncSetAttribute(sparse_attention_tc<D, AB, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)
                        : cudaFuncSetAttribute(sparse_attention_tc<D, AB, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  const long long total = static_cast<long long>(a.bh) * a.g.max_units;
  const int grid = static_cast<int>(total < num_sms() ? total : num_sms());
  if (split) sparse_attention_tc<D, AB, true><<<grid, kThreads, smem, stream>>>(qmap, a);
  else sparse_attention_tc<D, AB, false><<<grid, kThreads, smem, stream>>>(qmap, a);
  if (split) {  // the planner split key ranges: merge the parts
    const int rc = launch_status();
    if (rc) return rc;
    split_combine_kernel<D, AB><<<dim3(kSplitPieces, a.bh, D / 8), kUnitRows, 0, stream>>>(a);
  }
  return launch_status();
}

int check_shape(int bh, int sq, int sk, int d, int gq, int gk) {
  if (bh < 1 || bh > 65535 || sq < 0 || sk < 0 || gq < 1 || gk < 1) return kErrInvalidValue;
  if (d != 64 && d != 128) return kErrUnsupported;
  const PlanGeom g = plan_geom(sq, sk, gq, gk);
  // int32 positions (entries pack the end position << 8, so blocks < 2^23),
  // unit indices and per-head offsets
  if (g.blocks >= (1LL << 23) || static_cast<long long>(bh) * g.max_units > 2147483647LL ||
      g.stride > 2147483647LL)
    return kErrUnsupported;
  return kOk;
}

}  // namespace

int launch_attention_plan(const uint8_t* map, const int* q_sizes, const int* k_sizes, void* k_blocks,
                          void* v_blocks, int* ws, int bh, int sq, int sk, int d, int gq, int gk,
                          cudaStream_t stream) {
  int rc = check_shape(bh, sq, sk, d, gq, gk);
  if (rc) return rc;
  if ((k_blocks == nullptr) != (v_blocks == nullptr)) return kErrInvalidValue;
  if ((reinterpret_cast<uintptr_t>(ws) | reinterpret_cast<uintptr_t>(k_blocks) | reinterpret_cast<uintptr_t>(v_blocks)) & 15)
    return kErrInvalidValue;
  const PlanGeom g = plan_geom(sq, sk, gq, gk);
  size_t smem = sizeof(int) * (2 * static_cast<size_t>(gk + 1) + 2 * static_cast<size_t>(gq) + 2 * g.max_units +
                               4 * static_cast<size_t>(gq + 1));
  if (smem > 200 * 1024) return kErrUnsupported;
  const size_t map_bytes = static_cast<size_t>(gq) * gk;
  const int map_in_smem = smem + map_bytes <= 160 * 1024 ? 1 : 0;
  if (map_in_smem) smem += map_bytes;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attn_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  // at least kPlanParts CTAs per head, more when there are few heads, so the
  // per-unit map scans fill the GPU
  const int parts = max(kPlanParts, min(64, num_sms() / bh));
  attn_plan_kernel<<<dim3(bh, parts), 1024, smem, stream>>>(map, q_sizes, k_sizes, ws, g, static_cast<unsigned char*>(k_blocks),
                                               static_cast<unsigned char*>(v_blocks), kKeyBlockRows * d * 2, map_in_smem,
                                               attention_split_parts(bh, sk));
  return launch_status();
}

int launch_pack_key_blocks(const void* k, const void* v, void* k_blocks, void* v_blocks, const int* ws, int bh,
                           int sq, int sk, int d, int gq, int gk, cudaStream_t stream) {
  int rc = check_shape(bh, sq, sk, d, gq, gk);
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(k_blocks) |
       reinterpret_cast<uintptr_t>(v_blocks)) & 15)
    return kErrInvalidValue;
  const PlanGeom g = plan_geom(sq, sk, gq, gk);
  const long long chunks = static_cast<long long>(bh) * sk * (d / 8);
  if (chunks == 0) return kOk;
  long long blocks = (chunks + 255) / 256;
  if (blocks > kNumSMs * 16) blocks = kNumSMs * 16;
  if (d == 128)
    pack_key_blocks_kernel<128><<<static_cast<int>(blocks), 256, 0, stream>>>(
        static_cast<const uint4*>(k), static_cast<const uint4*>(v), static_cast<unsigned char*>(k_blocks),
        static_cast<unsigned char*>(v_blocks), ws, g, bh, device_status_ptr());
  else
    pack_key_blocks_kernel<64><<<static_cast<int>(blocks), 256, 0, stream>>>(
        static_cast<const uint4*>(k), static_cast<const uint4*>(v), static_cast<unsigned char*>(k_blocks),
        static_cast<unsigned char*>(v_blocks), ws, g, bh, device_status_ptr());
  return launch_status();
}

int launch_attention_main(const void* q, const void* k_blocks, const void* v_blocks, const int* ws, void* out,
                          int bh, int sq, int sk, int d, int gq, int gk, int dtype, const int32_t* perm, int video,
                          cudaStream_t stream) {
  int rc = check_shape(bh, sq, sk, d, gq, gk);
  if (rc) return rc;
  if (dtype != 0 && dtype != 1) return kErrInvalidValue;
  if (sq == 0) return kOk;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_blocks) | reinterpret_cast<uintptr_t>(v_blocks) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(ws)) & 15)
    return kErrInvalidValue;
  AttnArgs a;
  a.ws = ws;
  a.kb = static_cast<const unsigned char*>(k_blocks);
  a.vb = static_cast<const unsigned char*>(v_blocks);
  a.out = out;
  a.perm = perm;
  a.g = plan_geom(sq, sk, gq, gk);
  a.bh = bh;
  a.out_rows = sq;
  a.video = perm ? video : 0;
  a.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(d)));
  a.status = device_status_ptr();
  if (d == 128) return dtype ? launch_main<128, 1>(q, a, stream) : launch_main<128, 0>(q, a, stream);
  return dtype ? launch_main<64, 1>(q, a, stream) : launch_main<64, 0>(q, a, stream);
}

}  // namespace peco

using namespace peco;

// Drop-in for peco/kernels/sparse_attention.cu:210-230.  The caller's
// workspace (the reference's size) is accepted for ABI compatibility; the
// plan and the key blocks live in stream-ordered scratch of this call.
extern "C" int peco_sparse_attention(const void* q, const void* k, const void* v, const uint8_t* selected,
                                     const int* q_sizes, const int* k_sizes, void* output, int* workspace, int bh,
                                     int sq, int sk, int d, int cq, int ck, int dtype, void* stream_ptr) {
  (void)workspace;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int rc = check_shape(bh, sq, sk, d, cq, ck);
  if (rc) return rc;
  if (dtype != 0 && dtype != 1) return kErrInvalidValue;
  if (sq == 0) return kOk;
  const PlanGeom g = plan_geom(sq, sk, cq, ck);
  const size_t ws_bytes = (static_cast<size_t>(bh) * g.stride * sizeof(int) + 255) & ~size_t(255);
  const size_t kb_bytes = static_cast<size_t>(bh) * g.blocks * kKeyBlockRows * d * 2;
  void* scratch = nullptr;
  cudaError_t e = cudaMallocAsync(&scratch, ws_bytes + 2 * kb_bytes, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  int* ws = static_cast<int*>(scratch);
  unsigned char* kb = static_cast<unsigned char*>(scratch) + ws_bytes;
  unsigned char* vb = kb + kb_bytes;
  rc = launch_attention_plan(selected, q_sizes, k_sizes, kb, vb, ws, bh, sq, sk, d, cq, ck, stream);
  if (!rc) rc = launch_pack_key_blocks(k, v, kb, vb, ws, bh, sq, sk, d, cq, ck, stream);
  if (!rc) rc = launch_attention_main(q, kb, vb, ws, output, bh, sq, sk, d, cq, ck, dtype, nullptr, 0, stream);
  e = cudaFreeAsync(scratch, stream);
  return rc ? rc : static_cast<int>(e);
}

extern "C" long long peco_attention_workspace_stride(int sq, int sk, int gq, int gk) {
  if (sq < 0 || sk < 0 || gq < 1 || gk < 1) return -1;
  return plan_geom(sq, sk, gq, gk).stride;
}

extern "C" long long peco_key_block_rows(int sk, int gk) {
  if (sk < 0 || gk < 1) return -1;
  return plan_geom(0, sk, 1, gk).blocks * kKeyBlockRows;
}

extern "C" int peco_attention_plan(const uint8_t* map, const int* q_sizes, const int* k_sizes, void* k_blocks,
                                   void* v_blocks, int* workspace, int bh, int sq, int sk, int d, int gq, int gk,
                                   void* stream) {
  return launch_attention_plan(map, q_sizes, k_sizes, k_blocks, v_blocks, workspace, bh, sq, sk, d, gq, gk,
                               static_cast<cudaStream_t>(stream));
}

extern "C" int peco_pack_key_blocks(const void* k, const void* v, void* k_blocks, void* v_blocks,
                                    const int* workspace, int bh, int sq, int sk, int d, int gq, int gk,
                                    void* stream) {
  return launch_pack_key_blocks(k, v, k_blocks, v_blocks, workspace, bh, sq, sk, d, gq, gk,
                                static_cast<cudaStream_t>(stream));
}

extern "C" int peco_sparse_attention_restore(const void* q, const void* k_blocks, const void* v_blocks,
                                             const int* workspace, void* output, int bh, int sq, int sk, int d,
                                             int gq, int gk, const int32_t* q_indices, int video, void* stream) {
  if (video < 0 || video > sq) return kErrInvalidValue;
  return launch_attention_main(q, k_blocks, v_blocks, workspace, output, bh, sq, sk, d, gq, gk, 1, q_indices, video,
                               static_cast<cudaStream_t>(stream));
}
