// Cluster-block-sparse attention on sm_100a tensor cores.
//
// Replaces the reference's WMMA kernel (peco/kernels/sparse_attention.cu:55-190):
// O = softmax(Q K^T / sqrt(D), masked by map[group(i), group(j)]) V, rows
// with no allowed key -> 0.
//
// Work unit: up to 128 query rows of ONE query group (all rows of a unit
// share one key set, so masking is per key column only).  For each unit the
// selected key groups become contiguous runs of the group-packed K/V; every
// run is padded to whole 8-row groups, 16 groups make a 128-key tile, and
// consecutive groups of a run are fetched by one TMA box of 8, 16, 32, 64 or
// 128 rows (rows past a run's end are masked).  Per tile t:
//   S[t%2]  = Q K^T          tcgen05.mma, A = Q (smem), B = K tile (smem)
//   P       = exp2(S*c - m)  4 softmax warps, thread = query row; online max
//                            with lazy rescale of O (only when the max grows
//                            by > 8 in log2 units); P overwrites S[t%2] in
//                            TMEM as 16-bit pairs
//   O[u%2] += P V            tcgen05.mma, A = P (TMEM), B = V tile (smem, MN-major)
// The MMA issuer runs one tile ahead (QK of tile t+1 before PV of tile t), so
// the tensor core computes the next scores while the softmax warps work on the
// current ones.  K and V tiles stream through a 6-slot ring (three tiles in
// flight), and O is double-buffered so a unit's epilogue overlaps the next
// unit's MMAs.
//
// CTAs are persistent (one per SM) and take units heaviest-first: the
// planner lists every head's text groups (which attend to every key) before
// its video clusters, and CTAs claim (unit, head) pairs in unit-major order
// from a work counter in the workspace.
//
// Warp roles: warp 0 = TMA producer and scheduler, warp 1 = MMA issuer (one
// thread) and TMEM owner, warps 2-5 = softmax + epilogue.  The epilogue can
// scatter rows through an inverse permutation (fusing peco/clustering.py:
// 127-136 into the output store).  Every wait is bounded (common.cuh); on
// expiry the CTA records kDevTimeout in the device status word and unwinds.
#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

constexpr int kBM = 128;       // query rows per unit
constexpr int kBN = 128;       // keys per tile
constexpr int kGroup = 8;      // rows per key group (the padding granule)
constexpr int kGroups = kBN / kGroup;
constexpr int kSlots = 6;      // K/V ring: slot of K(t) = 2t mod 6, V(t) = 2t+1 mod 6
constexpr int kRing = 8;       // tile-info ring depth
constexpr int kThreads = 192;  // 6 warps
constexpr int kHeights = 5;    // TMA box heights 8 << h rows, h = 0..4
constexpr uint32_t kTmemCols = 512;  // S0 | S1 | O0 | O1, 128 columns each

// tile-info flags
constexpr uint32_t kFirst = 1u, kLast = 2u, kEmpty = 4u, kEnd = 8u;

#ifdef PECO_ATTN_TRACE
// Debug builds record per-CTA progress: trace[cta*8 + slot] = value.
#define ATTN_TRACE(slot, value)                                                                   \
  do {                                                                                            \
    if (args.trace) {                                                                             \
      volatile unsigned* t_ = args.trace + static_cast<long long>(blockIdx.x) * 8;                \
      t_[slot] = (value);                                                                         \
      __threadfence_system();                                                                     \
    }                                                                                             \
  } while (0)
#else
#define ATTN_TRACE(slot, value) \
  do {                          \
  } while (0)
#endif

struct AttnArgs {
#ifdef PECO_ATTN_TRACE
  unsigned* trace;
#endif
  const uint8_t* map;      // [BH, GQ, GK]
  int* ws;                 // planner output, ws_stride ints per head
  void* out;               // [BH, out_rows, D]
  const int32_t* perm;     // optional [BH, video] inverse permutation for packed rows < video
  int bh, sq, sk, gq, gk, ws_stride, max_units;
  int out_rows;            // rows per head of the output tensor
  int video;               // packed rows below this index go through perm
  int dynamic_sched;       // claim units from the work counter (else a static stride)
  float scale_log2;        // log2(e) / sqrt(D)
  unsigned* status;
};

// TMA descriptors: Q (128-row boxes) and K/V with box heights 8 << h.
struct AttnMaps {
  CUtensorMap q;
  CUtensorMap k[kHeights];
  CUtensorMap v[kHeights];
};

struct TileInfo {
  uint32_t mask[4];        // key rows of the tile that are valid
  int unit;                // virtual unit index (local * BH + head)
  uint32_t flags;
};

struct __align__(8) Shared {
  uint64_t q_full, q_empty;
  uint64_t slot_full[kSlots], slot_empty[kSlots];
  uint64_t s_full[2], s_free[2], p_full[2];
  uint64_t o_full[2], o_free[2];
  uint64_t info_full[kRing], info_empty[kRing];
  TileInfo info[kRing];
  uint32_t tmem_base;
  int abort_flag;
};

// Operand tiles (Q, K, V) share one layout: two 64-column panels of 128 rows
// x 128 bytes (16 KB each, 128-byte swizzle), 8-row groups 1 KB apart.
template <int D>
struct Layout {
  static constexpr int kTileBytes = kBN * D * 2;
  static constexpr int kPanel = kBN * 128;
  static constexpr int kQ0 = 0;
  static constexpr int kSlot0 = kTileBytes;
  static constexpr int kShared = kSlot0 + kSlots * kTileBytes;
  static constexpr int kSmem = 1024 + kShared + static_cast<int>(sizeof(Shared));
};

__device__ __forceinline__ int* work_counter(const AttnArgs& a) {
  return a.ws + static_cast<long long>(a.bh - 1) * a.ws_stride + (a.ws_stride - 1);
}

// ---------------------------------------------------------------------------
// planner: clamped group prefixes and the unit list of every head
// ---------------------------------------------------------------------------
// ws per head: [0] = unit count, [1 .. gk+1] = key group starts, then
// 3 ints per unit (q_start, q_count, q_group).  Group extents are clamped the
// way the reference's work map clamps them (sparse_attention.cu:25-31):
// start_g = min(S, sum_{g'<g} max(0, size_g')).  Units of later groups come
// first, so the text groups (which attend to every key) start early.
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

// dynamic smem: 2 * gq ints (clamped start and size of every query group)
__global__ void __launch_bounds__(1024) attn_plan_kernel(const int* __restrict__ q_sizes, const int* __restrict__ k_sizes,
                                                         int* __restrict__ ws, int gq, int gk, int sq, int sk,
                                                         int ws_stride, int zero_counter) {
  extern __shared__ int plan_sm[];
  int* gstart = plan_sm;
  int* gcount = plan_sm + gq;
  __shared__ long long tmp[32];
  __shared__ long long carry;
  const int head = blockIdx.x;
  int* w = ws + static_cast<long long>(head) * ws_stride;
  int* kp = w + 1;
  int* units = w + 2 + gk;
  const int* qs = q_sizes + static_cast<long long>(head) * gq;
  const int* ks = k_sizes + static_cast<long long>(head) * gk;
  const int last = blockDim.x - 1;
  if (threadIdx.x == 0) {
    carry = 0;
    kp[0] = 0;
    // work counter of the persistent attention kernel (last int of the last head)
    if (zero_counter && head == gridDim.x - 1) w[ws_stride - 1] = 0;
  }
  __syncthreads();
  for (int c0 = 0; c0 < gk; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    const long long v = c < gk ? max(0, ks[c]) : 0;
    const long long pre = carry + block_exclusive_scan(v, tmp);
    if (c < gk) kp[c + 1] = static_cast<int>(min(static_cast<long long>(sk), pre + v));
    __syncthreads();
    if (threadIdx.x == last) carry = pre + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int g0 = 0; g0 < gq; g0 += blockDim.x) {
    const int g = g0 + threadIdx.x;
    const long long v = g < gq ? max(0, qs[g]) : 0;
    const long long pre = carry + block_exclusive_scan(v, tmp);
    if (g < gq) {
      const long long s0 = min(static_cast<long long>(sq), pre), s1 = min(static_cast<long long>(sq), pre + v);
      gstart[g] = static_cast<int>(s0);
      gcount[g] = static_cast<int>(s1 - s0);
    }
    __syncthreads();
    if (threadIdx.x == last) carry = pre + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int o0 = 0; o0 < gq; o0 += blockDim.x) {
    const int o = o0 + threadIdx.x;
    const int g = gq - 1 - o;
    const int n = o < gq ? gcount[g] : 0;
    const long long nu = (n + kBM - 1) / kBM;
    const long long u0 = carry + block_exclusive_scan(nu, tmp);
    for (int i = 0; i < nu; ++i) {
      int* rec = units + 3 * (u0 + i);
      rec[0] = gstart[g] + i * kBM;
      rec[1] = min(kBM, n - i * kBM);
      rec[2] = g;
    }
    __syncthreads();
    if (threadIdx.x == last) carry = u0 + nu;
    __syncthreads();
  }
  if (threadIdx.x == 0) w[0] = static_cast<int>(carry);
}

// ---------------------------------------------------------------------------
// main kernel (persistent)
// ---------------------------------------------------------------------------
template <int D, int AB>  // AB: 0 = fp16, 1 = bf16
__global__ void __launch_bounds__(kThreads, 1) sparse_attention_tc(const __grid_constant__ AttnMaps maps,
                                                                  const AttnArgs args) {
  using L = Layout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared& sh = *reinterpret_cast<Shared*>(base + L::kShared);
  volatile int* abort_flag = &sh.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long total_units = static_cast<long long>(args.bh) * args.max_units;

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    mbar_init(&sh.q_empty, 1);
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sh.slot_full[i], 1);
      mbar_init(&sh.slot_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.s_full[i], 1);
      mbar_init(&sh.s_free[i], 1);
      mbar_init(&sh.p_full[i], 4);
      mbar_init(&sh.o_full[i], 1);
      mbar_init(&sh.o_free[i], 4);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&sh.info_full[i], 1);
      mbar_init(&sh.info_empty[i], 5);  // MMA thread + 4 softmax warps
    }
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  // K/V rows of padding groups are never loaded: zero the ring once so the
  // tensor core only ever sees finite values there
  for (int i = threadIdx.x; i < kSlots * L::kTileBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(base + L::kSlot0)[i] = make_uint4(0, 0, 0, 0);
  fence_async_smem();
  if (threadIdx.x == 0) ATTN_TRACE(0, 1);
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&maps.q);
      for (int h = 0; h < kHeights; ++h) {
        prefetch_tensormap(&maps.k[h]);
        prefetch_tensormap(&maps.v[h]);
      }
    }
    bool ok = true;
    int tile = 0;      // tiles issued by this CTA
    int entry = 0;     // info entries pushed
    int qloads = 0;    // Q tiles loaded
    int claims = 0;
    auto push_info = [&](const uint32_t (&mask)[4], int unit, uint32_t flags) {
      const int slot = entry % kRing;
      if (ok && entry >= kRing) ok = mbar_wait_warp(&sh.info_empty[slot], ((entry / kRing) - 1) & 1, abort_flag, args.status);
      if (lane == 0 && ok) {
        TileInfo& ti = sh.info[slot];
        ti.mask[0] = mask[0];
        ti.mask[1] = mask[1];
        ti.mask[2] = mask[2];
        ti.mask[3] = mask[3];
        ti.unit = unit;
        ti.flags = flags;
        mbar_arrive(&sh.info_full[slot]);
      }
      __syncwarp();
      ++entry;
    };
    // Fill ring item ``item`` (K or V of a tile) with the pending groups: lane
    // g < ngroups holds the global row of group g; runs of groups with
    // consecutive rows become power-of-two boxes issued by their first lane.
    auto fill_slot = [&](int item, const CUtensorMap* hmaps, int grow, int ngroups) {
      const int sl = item % kSlots, fill = item / kSlots;
      if (ok && fill > 0) ok = mbar_wait_warp(&sh.slot_empty[sl], (fill - 1) & 1, abort_flag, args.status);
      if (!ok) return;
      if (lane == 0) mbar_arrive_expect_tx(&sh.slot_full[sl], static_cast<uint32_t>(ngroups) * kGroup * D * 2);
      __syncwarp();
      const int prev = __shfl_up_sync(0xffffffffu, grow, 1);
      const bool cont = lane > 0 && lane < ngroups && grow == prev + kGroup;
      const unsigned cmask = __ballot_sync(0xffffffffu, cont);
      if (lane < ngroups && !cont) {
        // this lane starts a segment: count its groups, then issue its boxes
        int n = 1;
        while (lane + n < ngroups && ((cmask >> (lane + n)) & 1u)) ++n;
        int g = lane, row = grow;
        for (int h = kHeights - 1; h >= 0; --h) {
          const int cnt = 1 << h;
          while (n >= cnt) {
            unsigned char* dst = base + L::kSlot0 + sl * L::kTileBytes + g * (kGroup * 128);
#pragma unroll
            for (int p = 0; p < D / 64; ++p) tma_load_2d(dst + p * L::kPanel, &hmaps[h], 64 * p, row, &sh.slot_full[sl]);
            g += cnt;
            row += cnt * kGroup;
            n -= cnt;
          }
        }
      }
      __syncwarp();
    };
    for (;;) {
      // ---- claim a unit
      long long v = 0;
      if (args.dynamic_sched) {
        int got = 0;
        if (lane == 0) got = atomicAdd(work_counter(args), 1);
        v = __shfl_sync(0xffffffffu, got, 0);
      } else {
        v = static_cast<long long>(blockIdx.x) + static_cast<long long>(claims) * gridDim.x;
        ++claims;
      }
      if (v >= total_units || !ok) break;
      const int head = static_cast<int>(v % args.bh);
      const int local = static_cast<int>(v / args.bh);
      const int* w = args.ws + static_cast<long long>(head) * args.ws_stride;
      if (local >= w[0]) continue;
      const int* kp = w + 1;
      const int* rec = w + 2 + args.gk + 3 * local;
      const int q_start = rec[0], qg = rec[2];
      const uint8_t* map_row = args.map + (static_cast<long long>(head) * args.gq + qg) * args.gk;
      const long long krow0 = static_cast<long long>(head) * args.sk;

      // ---- stream the unit's key runs as 8-row groups grouped into tiles
      int grow = 0, gvalid = 0;  // lane g holds group g of the pending tile
      int ngroups = 0;
      int utiles = 0;
      int run_s = 0, run_e = 0;
      bool have_run = false;
      auto emit_tile = [&](bool last) {
        fill_slot(2 * tile, maps.k, grow, ngroups);
        fill_slot(2 * tile + 1, maps.v, grow, ngroups);
        if (utiles == 0) {
          // first tile of a non-empty unit: its Q tile, once the previous
          // unit's last QK has released the buffer (its K/V are already in flight)
          if (ok && qloads > 0) ok = mbar_wait_warp(&sh.q_empty, (qloads - 1) & 1, abort_flag, args.status);
          if (lane == 0 && ok) {
            mbar_arrive_expect_tx(&sh.q_full, L::kTileBytes);
#pragma unroll
            for (int p = 0; p < D / 64; ++p)
              tma_load_2d(base + L::kQ0 + p * L::kPanel, &maps.q, 64 * p,
                          static_cast<int>(static_cast<long long>(head) * args.sq + q_start), &sh.q_full);
          }
          __syncwarp();
          ++qloads;
        }
        const unsigned bits = lane < ngroups ? ((gvalid >= 8) ? 0xffu : ((1u << gvalid) - 1u)) : 0u;
        uint32_t word[4] = {0, 0, 0, 0};
#pragma unroll
        for (int b = 0; b < kGroups; ++b) word[b >> 2] |= __shfl_sync(0xffffffffu, bits, b) << (8 * (b & 3));
        push_info(word, static_cast<int>(v), (utiles == 0 ? kFirst : 0u) | (last ? kLast : 0u));
        ++tile;
        ++utiles;
        ngroups = 0;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (lane == 0) ATTN_TRACE(1, 0x100u + tile);
      };
      auto add_group = [&](int row, int valid) {
        if (ngroups == kGroups) emit_tile(false);
        if (lane == ngroups) {
          grow = row;
          gvalid = valid;
        }
        ++ngroups;
      };
      auto flush_run = [&]() {
        for (int r = run_s; r < run_e && ok; r += kGroup) add_group(static_cast<int>(krow0 + r), min(kGroup, run_e - r));
      };
      for (int c0 = 0; c0 < args.gk && ok; c0 += 32) {
        const int c = c0 + lane;
        int s = 0, e = 0;
        bool sel = false;
        if (c < args.gk) {
          s = kp[c];
          e = kp[c + 1];
          sel = map_row[c] != 0 && e > s;
        }
        unsigned m = __ballot_sync(0xffffffffu, sel);
        while (m && ok) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          const int gs = __shfl_sync(0xffffffffu, s, b);
          const int ge = __shfl_sync(0xffffffffu, e, b);
          if (have_run && gs == run_e) {
            run_e = ge;
          } else {
            if (have_run) flush_run();
            run_s = gs;
            run_e = ge;
            have_run = true;
          }
        }
        if (*abort_flag) ok = false;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
      if (have_run && ok) flush_run();
      if (!ok) break;
      if (utiles == 0 && ngroups == 0) {
        const uint32_t zero[4] = {0, 0, 0, 0};
        push_info(zero, static_cast<int>(v), kEmpty);  // no key at all: rows are zero
      } else {
        emit_tile(true);
      }
    }
    const uint32_t zero[4] = {0, 0, 0, 0};
    push_info(zero, -1, kEnd);
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t idesc_qk = instr_desc(128, kBN, AB, false, false);
      constexpr uint32_t idesc_pv = instr_desc(128, D, AB, false, true);
      bool ok = true;
      int entry = 0, t = 0, qloads = 0, ounits = 0;
      int cur = -1;           // tile whose P.V is pending
      uint32_t cur_flags = 0;
      int cur_oslot = 0;
      auto issue_pv = [&]() {
        const int b = cur & 1, item = 2 * cur + 1, sl = item % kSlots;
        ok = mbar_wait(&sh.p_full[b], (cur >> 1) & 1, abort_flag, args.status);
        if (ok) ok = mbar_wait(&sh.slot_full[sl], (item / kSlots) & 1, abort_flag, args.status);
        if (!ok) return;
        tc_fence_after();
        const uint32_t va = smem_u32(base + L::kSlot0 + sl * L::kTileBytes);
        const uint32_t o_addr = tmem + 256 + cur_oslot * 128;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bdesc = smem_desc(va + kk * 2 * 1024, L::kPanel, 1024);
          umma_ts(o_addr, tmem + b * 128 + kk * 8, bdesc, idesc_pv, ((cur_flags & kFirst) && kk == 0) ? 0u : 1u);
        }
        umma_commit(&sh.s_free[b]);
        umma_commit(&sh.slot_empty[sl]);
        if (cur_flags & kLast) umma_commit(&sh.o_full[cur_oslot]);
        ATTN_TRACE(2, 0x200u + cur);
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
          ok = mbar_wait(&sh.q_full, qloads & 1, abort_flag, args.status);
          ++qloads;
        }
        if (ok) ok = mbar_wait(&sh.slot_full[sl], (item / kSlots) & 1, abort_flag, args.status);
        if (ok && t >= 2) ok = mbar_wait(&sh.s_free[b], ((t >> 1) - 1) & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(base + L::kQ0);
        const uint32_t ka = smem_u32(base + L::kSlot0 + sl * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kPanel + (kk & 3) * 32;
          umma_ss(tmem + b * 128, smem_desc(qa + off, 16, 1024), smem_desc(ka + off, 16, 1024), idesc_qk,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(&sh.s_full[b]);
        umma_commit(&sh.slot_empty[sl]);
        if (fl & kLast) umma_commit(&sh.q_empty);
        ATTN_TRACE(2, 0x100u + t);
        // ---- O += P V for the previous tile
        if (cur >= 0) {
          issue_pv();
          if (!ok) break;
        }
        cur = t;
        cur_flags = fl;
        if (fl & kFirst) {
          cur_oslot = ounits & 1;
          if (ounits >= 2) ok = mbar_wait(&sh.o_free[cur_oslot], ((ounits >> 1) - 1) & 1, abort_flag, args.status);
          ++ounits;
          if (!ok) break;
        }
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
    const int r = quarter * 32 + lane;             // query row within the unit
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    int entry = 0, t = 0, ounits = 0, oslot = 0;
    // write this thread's row of unit v: O/l, or zero when ``zero``
    auto write_row = [&](int v, bool have_o, float inv) {
      const int head = v % args.bh, local = v / args.bh;
      const int* rec = args.ws + static_cast<long long>(head) * args.ws_stride + 2 + args.gk + 3 * local;
      const int q_start = rec[0], q_count = rec[1];
      T* dst = nullptr;
      if (r < q_count) {
        const int prow = q_start + r;
        long long orow = prow;
        if (args.perm && prow < args.video) orow = args.perm[static_cast<long long>(head) * args.video + prow];
        if (orow < 0 || orow >= args.out_rows) record_status(args.status, kDevBadIndex);
        else dst = static_cast<T*>(args.out) + (static_cast<long long>(head) * args.out_rows + orow) * D;
      }
      __syncwarp();
      if (have_o) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t vv[32];
          tmem_ld32_sync(tmem + 256 + oslot * 128 + lane_off + c * 32, vv);
          if (dst) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 pk;
              uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = __uint_as_float(vv[j + 2 * e]) * inv, bb = __uint_as_float(vv[j + 2 * e + 1]) * inv;
                pw[e] = AB ? pack_bf16x2(a, bb) : pack_f16x2(a, bb);
              }
              reinterpret_cast<uint4*>(dst)[(c * 32 + j) / 8] = pk;
            }
          }
        }
      } else if (dst) {
#pragma unroll
        for (int c = 0; c < D / 8; ++c) reinterpret_cast<uint4*>(dst)[c] = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    };
    for (;;) {
      const int slot = entry % kRing;
      ok = mbar_wait_warp(&sh.info_full[slot], (entry / kRing) & 1, abort_flag, args.status);
      if (!ok) break;
      const TileInfo ti = sh.info[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.info_empty[slot]);
      ++entry;
      if (ti.flags & kEnd) break;
      if (ti.flags & kEmpty) {
        write_row(ti.unit, false, 0.0f);
        continue;
      }
      if (ti.flags & kFirst) {
        m = -INFINITY;
        l = 0.0f;
        oslot = ounits & 1;
        ++ounits;
      }
      const int b = t & 1;
      ok = mbar_wait_warp(&sh.s_full[b], (t >> 1) & 1, abort_flag, args.status);
      if (!ok) break;
      tc_fence_after();
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t vv[32];
        tmem_ld32_sync(tmem + b * 128 + lane_off + c * 32, vv);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[c * 32 + j] = __uint_as_float(vv[j]);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kBN; ++j) {
        const bool valid = (ti.mask[j >> 5] >> (j & 31)) & 1u;
        s[j] = valid ? s[j] * args.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[j]);
      }
      // grow the running max lazily (only by > 8 in log2 units); rescaling O
      // is warp-collective (tcgen05.ld/st are .sync.aligned) and needs the
      // previous tile's P.V to be complete
      const bool grow = (mx > m + 8.0f) || (m == -INFINITY && mx > -INFINITY);
      const bool rescale_me = grow && m != -INFINITY;
      if (__any_sync(0xffffffffu, rescale_me)) {
        ok = mbar_wait_warp(&sh.s_free[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
        const float f = rescale_me ? exp2f(m - mx) : 1.0f;
        l *= f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t vv[32];
          tmem_ld32_sync(tmem + 256 + oslot * 128 + lane_off + c * 32, vv);
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            lo[j] = __float_as_uint(__uint_as_float(vv[j]) * f);
            hi[j] = __float_as_uint(__uint_as_float(vv[16 + j]) * f);
          }
          tmem_st16(tmem + 256 + oslot * 128 + lane_off + c * 32, lo);
          tmem_st16(tmem + 256 + oslot * 128 + lane_off + c * 32 + 16, hi);
        }
      }
      if (grow) m = mx;
      const float mref = (m == -INFINITY) ? 0.0f : m;
      float sum = 0.0f;
      uint32_t packed[kBN / 2];
#pragma unroll
      for (int j = 0; j < kBN; j += 2) {
        const float p0 = exp2f(s[j] - mref);
        const float p1 = exp2f(s[j + 1] - mref);
        sum += p0 + p1;
        packed[j >> 1] = AB ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
      }
      l += sum;
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t part[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) part[j] = packed[c * 16 + j];
        tmem_st16(tmem + b * 128 + lane_off + c * 16, part);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.p_full[b]);
      if (lane == 0) ATTN_TRACE(3 + quarter, 0x300u + t);
      ++t;
      if (ti.flags & kLast) {
        // epilogue of the unit: O[oslot] is final once its last P.V completes
        ok = mbar_wait_warp(&sh.o_full[oslot], ((ounits - 1) >> 1) & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
        write_row(ti.unit, true, l > 0.0f ? 1.0f / l : 0.0f);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.o_free[oslot]);
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) ATTN_TRACE(0, 3);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

#ifdef PECO_ATTN_TRACE
unsigned* g_attn_trace = nullptr;
#endif

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

template <int D, int AB>
int launch_main(const void* q, const void* k, const void* v, const AttnArgs& a, cudaStream_t stream) {
  AttnMaps maps;
  if (!make_rows_map(&maps.q, q, static_cast<long long>(a.bh) * a.sq, D, kBM, AB)) return kErrTensorMap;
  for (int h = 0; h < kHeights; ++h) {
    if (!make_rows_map(&maps.k[h], k, static_cast<long long>(a.bh) * a.sk, D, kGroup << h, AB) ||
        !make_rows_map(&maps.v[h], v, static_cast<long long>(a.bh) * a.sk, D, kGroup << h, AB))
      return kErrTensorMap;
  }
  const int smem = Layout<D>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(sparse_attention_tc<D, AB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  const long long total = static_cast<long long>(a.bh) * a.max_units;
  const int grid = static_cast<int>(total < num_sms() ? total : num_sms());
  sparse_attention_tc<D, AB><<<grid, kThreads, smem, stream>>>(maps, a);
  return launch_status();
}

}  // namespace

int launch_sparse_attention(const void* q, const void* k, const void* v, const uint8_t* map, const int* q_sizes,
                            const int* k_sizes, void* out, int* ws, int ws_stride, int bh, int sq, int sk, int d,
                            int gq, int gk, int dtype, const int32_t* perm, int video, cudaStream_t stream) {
  if (bh < 1 || bh > 65535 || sq < 0 || sk < 0 || gq < 1 || gk < 1 || (dtype != 0 && dtype != 1))
    return kErrInvalidValue;
  if (d != 64 && d != 128) return kErrUnsupported;
  if (sq == 0) return kOk;
  const long long max_units = (static_cast<long long>(sq) + kBM - 1) / kBM + gq;
  const long long need = 2 + gk + 3 * max_units;
  if (need > ws_stride) return kErrWorkspace;
  if (static_cast<long long>(bh) * max_units > 2147483647LL) return kErrUnsupported;
  const size_t plan_smem = 2 * sizeof(int) * static_cast<size_t>(gq);
  if (plan_smem > 200 * 1024) return kErrUnsupported;
  if (plan_smem > 48 * 1024)
    cudaFuncSetAttribute(attn_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan_smem));
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return kErrInvalidValue;
  // the work counter takes the last int of the last head's region when the
  // workspace has room for it; otherwise CTAs take units with a fixed stride
  const int dynamic = ws_stride >= need + 1 ? 1 : 0;
  attn_plan_kernel<<<bh, 1024, plan_smem, stream>>>(q_sizes, k_sizes, ws, gq, gk, sq, sk, ws_stride, dynamic);
  int rc = launch_status();
  if (rc) return rc;
  AttnArgs a;
#ifdef PECO_ATTN_TRACE
  a.trace = g_attn_trace;
#endif
  a.map = map;
  a.ws = ws;
  a.out = out;
  a.perm = perm;
  a.bh = bh;
  a.sq = sq;
  a.sk = sk;
  a.gq = gq;
  a.gk = gk;
  a.ws_stride = ws_stride;
  a.max_units = static_cast<int>(max_units);
  a.out_rows = sq;
  a.video = perm ? video : 0;
  a.dynamic_sched = dynamic;
  a.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(d)));
  a.status = device_status_ptr();
  if (d == 128) return dtype ? launch_main<128, 1>(q, k, v, a, stream) : launch_main<128, 0>(q, k, v, a, stream);
  return dtype ? launch_main<64, 1>(q, k, v, a, stream) : launch_main<64, 0>(q, k, v, a, stream);
}

// Workspace ints per head needed by launch_sparse_attention (the last one
// of the last head holds the work counter).
long long attention_ws_stride(int sq, int gq, int gk) {
  const long long max_units = (static_cast<long long>(sq) + kBM - 1) / kBM + gq;
  return 3 + gk + 3 * max_units;
}

}  // namespace peco

// Drop-in for peco/kernels/sparse_attention.cu:210-230.  Workspace: int32
// BH * (CK + 2 + 3 * (ceil(SQ/16) + CQ)), the reference's size.
extern "C" int peco_sparse_attention(const void* q, const void* k, const void* v, const uint8_t* selected,
                                     const int* q_sizes, const int* k_sizes, void* output, int* workspace, int bh,
                                     int sq, int sk, int d, int cq, int ck, int dtype, void* stream) {
  const long long cap = (static_cast<long long>(sq) + 15) / 16 + cq;
  const long long stride = ck + 2 + 3 * cap;
  if (stride > 2147483647LL) return peco::kErrInvalidValue;
  return peco::launch_sparse_attention(q, k, v, selected, q_sizes, k_sizes, output, workspace,
                                       static_cast<int>(stride), bh, sq, sk, d, cq, ck, dtype, nullptr, 0,
                                       static_cast<cudaStream_t>(stream));
}

extern "C" long long peco_attention_workspace_stride(int sq, int gq, int gk) {
  return peco::attention_ws_stride(sq, gq, gk);
}

extern "C" int peco_sparse_attention_restore(const void* q, const void* k, const void* v, const uint8_t* map,
                                             const int* q_sizes, const int* k_sizes, void* output, int* workspace,
                                             int bh, int sq, int sk, int d, int gq, int gk, const int32_t* q_indices,
                                             int video, void* stream) {
  const long long stride = peco::attention_ws_stride(sq, gq, gk);
  if (stride > 2147483647LL || video < 0 || video > sq) return peco::kErrInvalidValue;
  return peco::launch_sparse_attention(q, k, v, map, q_sizes, k_sizes, output, workspace, static_cast<int>(stride), bh,
                                       sq, sk, d, gq, gk, 1, q_indices, video, static_cast<cudaStream_t>(stream));
}
