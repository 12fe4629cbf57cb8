// Cluster-block-sparse attention on sm_100a tensor cores.
//
// Replaces the reference's WMMA kernel (peco/kernels/sparse_attention.cu:55-190):
// O = softmax(Q K^T / sqrt(D), masked by map[group(i), group(j)]) V, rows
// with no allowed key -> 0.
//
// Work unit: up to 128 query rows of ONE query group (all rows of a unit
// share one key set, so masking is per key column only).  For each unit the
// selected key groups become contiguous runs of the group-packed K/V; runs
// are streamed as 8-row TMA boxes into 128-key tiles (rows of a box past the
// run's end are masked).  Per tile:
//   S = Q K^T           tcgen05.mma, A = Q (smem), B = K tile (smem), S in TMEM
//   P = exp2(S*c - m)   4 softmax warps, thread = query row, online max with
//                       lazy rescale of O (only when the max grows by > 8 in
//                       log2 units); P written back to TMEM as 16-bit pairs
//   O += P V            tcgen05.mma, A = P (TMEM), B = V tile (smem, MN-major)
// Warp roles: warp 0 = TMA producer, warp 1 = MMA issuer (one thread) and
// TMEM owner, warps 2-5 = softmax + epilogue.  Two CTAs share an SM (256
// TMEM columns and ~100 KB smem each) so one CTA's softmax overlaps the
// other's MMAs.  The epilogue optionally scatters rows through an inverse
// permutation (fusing peco/clustering.py:127-136 into the output store).
//
// Every wait is bounded (common.cuh); on expiry the CTA records kDevTimeout
// in the device status word, drains what it issued and exits.
#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

constexpr int kBM = 128;       // query rows per unit
constexpr int kBN = 128;       // keys per tile
constexpr int kBox = 8;        // rows per TMA box
constexpr int kBoxes = kBN / kBox;
constexpr int kRing = 4;       // mask ring depth
constexpr int kThreads = 192;  // 6 warps
constexpr uint32_t kTmemCols = 256;

#ifdef PECO_ATTN_TRACE
// Debug builds record per-CTA progress: trace[cta*8 + role] = stage code.
#define ATTN_TRACE(slot, value)                                                                   \
  do {                                                                                            \
    if (args.trace) {                                                                             \
      volatile unsigned* t_ = args.trace + (static_cast<long long>(blockIdx.y) * gridDim.x + blockIdx.x) * 8; \
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
  const int* ws;           // planner output, ws_stride ints per head
  void* out;               // [BH, SO, D]
  const int32_t* perm;     // optional [BH, video] inverse permutation for packed rows < video
  int sq, sk, gq, gk, ws_stride;
  int out_rows;            // rows per head of the output tensor
  int video;               // packed rows below this index go through perm
  float scale_log2;        // log2(e) / sqrt(D)
  unsigned* status;
};

struct __align__(8) Shared {
  uint64_t q_full, k_full, k_empty, v_full, v_empty, s_full, p_full, pv_done;
  uint64_t mask_full[kRing], mask_empty[kRing];
  uint32_t mask[kRing][4];
  uint32_t flags[kRing];   // bit0: last tile, bit1: unit has no keys
  uint32_t tmem_base;
  int abort_flag;
};

template <int D>
struct Layout {
  static constexpr int kTileBytes = kBN * D * 2;   // K or V tile, also the Q tile
  static constexpr int kBoxBytes = kBox * D * 2;   // one 8-row box (D/64 panels of 1 KB)
  static constexpr int kQPanel = kBM * 128;        // Q panel: 128 rows x 128 B
  static constexpr int kSmem = 1024 + 3 * kTileBytes + static_cast<int>(sizeof(Shared));
};

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
                                                         int ws_stride) {
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
// main kernel
// ---------------------------------------------------------------------------
template <int D, int AB>  // AB: 0 = fp16, 1 = bf16
__global__ void __launch_bounds__(kThreads, 2) sparse_attention_tc(const __grid_constant__ CUtensorMap tmap_q,
                                                                  const __grid_constant__ CUtensorMap tmap_k,
                                                                  const __grid_constant__ CUtensorMap tmap_v,
                                                                  const AttnArgs args) {
  using L = Layout<D>;
  const int head = blockIdx.y;
  const int* w = args.ws + static_cast<long long>(head) * args.ws_stride;
  const int nunits = w[0];
  if (static_cast<int>(blockIdx.x) >= nunits) return;
  const int* kp = w + 1;
  const int* unit = w + 2 + args.gk + 3 * blockIdx.x;
  const int q_start = unit[0], q_count = unit[1], qg = unit[2];

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* q_tile = base;
  unsigned char* k_tile = base + L::kTileBytes;
  unsigned char* v_tile = base + 2 * L::kTileBytes;
  Shared& sh = *reinterpret_cast<Shared*>(base + 3 * L::kTileBytes);
  volatile int* abort_flag = &sh.abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    mbar_init(&sh.k_full, 1);
    mbar_init(&sh.k_empty, 1);
    mbar_init(&sh.v_full, 1);
    mbar_init(&sh.v_empty, 1);
    mbar_init(&sh.s_full, 1);
    mbar_init(&sh.p_full, 4);
    mbar_init(&sh.pv_done, 1);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&sh.mask_full[i], 1);
      mbar_init(&sh.mask_empty[i], 5);  // MMA thread + 4 softmax warps
    }
    sh.abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 0) ATTN_TRACE(0, 1);
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  if (threadIdx.x == 0) ATTN_TRACE(0, 2);
  const uint32_t tmem_s = tmem;          // S: columns [0,128); P aliases [0,64)
  const uint32_t tmem_o = tmem + 128;    // O: columns [128, 128+D)

  const uint8_t* map_row = args.map + (static_cast<long long>(head) * args.gq + qg) * args.gk;
  const long long krow0 = static_cast<long long>(head) * args.sk;

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&tmap_q);
      prefetch_tensormap(&tmap_k);
      prefetch_tensormap(&tmap_v);
      mbar_arrive_expect_tx(&sh.q_full, L::kTileBytes);
#pragma unroll
      for (int p = 0; p < D / 64; ++p)
        tma_load_2d(q_tile + p * L::kQPanel, &tmap_q, 64 * p, static_cast<int>(static_cast<long long>(head) * args.sq + q_start), &sh.q_full);
    }
    // pending tile: box rows and valid counts live in lanes 0..15
    int box_row = 0, box_valid = 0;  // for lane == box index
    int nbox = 0;                    // boxes collected in the pending tile
    int tile = 0;
    bool ok = true;
    int run_s = 0, run_e = 0;        // pending merged run (lane-uniform)
    auto emit_tile = [&](bool last) {
      // pad unused boxes with in-bounds rows of this head, fully masked
      if (lane >= nbox && lane < kBoxes) {
        box_row = static_cast<int>(krow0);
        box_valid = 0;
      }
      const int slot = tile % kRing;
      const uint32_t ph = (tile / kRing) & 1;
      if (ok && tile >= kRing) ok = mbar_wait_warp(&sh.mask_empty[slot], ph ^ 1, abort_flag, args.status);
      unsigned vm = 0;
      // mask words: bit j of word i -> key row 32 i + j valid
      {
        const unsigned bits = (box_valid >= 8) ? 0xffu : ((1u << box_valid) - 1u);
        unsigned word[4] = {0, 0, 0, 0};
#pragma unroll
        for (int b = 0; b < kBoxes; ++b) {
          const unsigned bb = __shfl_sync(0xffffffffu, bits, b);
          word[b >> 2] |= bb << (8 * (b & 3));
        }
        vm = word[0];
        if (lane == 0 && ok) {
          sh.mask[slot][0] = word[0];
          sh.mask[slot][1] = word[1];
          sh.mask[slot][2] = word[2];
          sh.mask[slot][3] = word[3];
          sh.flags[slot] = last ? 1u : 0u;
        }
      }
      (void)vm;
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&sh.mask_full[slot]);
      // K boxes
      if (ok && tile > 0) ok = mbar_wait_warp(&sh.k_empty, (tile - 1) & 1, abort_flag, args.status);
      if (lane == 0 && ok) mbar_arrive_expect_tx(&sh.k_full, L::kTileBytes);
      __syncwarp();
      if (ok && lane < kBoxes) {
#pragma unroll
        for (int p = 0; p < D / 64; ++p)
          tma_load_2d(k_tile + lane * L::kBoxBytes + p * 1024, &tmap_k, 64 * p, box_row, &sh.k_full);
      }
      // V boxes (the V tile is free once the previous P.V finished)
      if (ok && tile > 0) ok = mbar_wait_warp(&sh.v_empty, (tile - 1) & 1, abort_flag, args.status);
      if (lane == 0 && ok) mbar_arrive_expect_tx(&sh.v_full, L::kTileBytes);
      __syncwarp();
      if (ok && lane < kBoxes) {
#pragma unroll
        for (int p = 0; p < D / 64; ++p)
          tma_load_2d(v_tile + lane * L::kBoxBytes + p * 1024, &tmap_v, 64 * p, box_row, &sh.v_full);
      }
      ++tile;
      nbox = 0;
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (lane == 0) ATTN_TRACE(1, 0x100u + tile);
    };
    auto add_box = [&](int row, int valid) {
      if (nbox == kBoxes) emit_tile(false);
      if (lane == nbox) {
        box_row = row;
        box_valid = valid;
      }
      ++nbox;
    };
    auto flush_run = [&]() {
      for (int r = run_s; r < run_e && ok; r += kBox) add_box(static_cast<int>(krow0 + r), min(kBox, run_e - r));
    };
    bool have_run = false;
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
    if (ok) {
      if (tile == 0 && nbox == 0) {
        // no key at all: announce an empty unit
        if (lane == 0) {
          sh.flags[0] = 3u;
          mbar_arrive(&sh.mask_full[0]);
        }
      } else {
        emit_tile(true);
      }
    }
    // drain: wait for the loads this warp issued before the CTA exits
    if (tile > 0) {
      mbar_wait_warp(&sh.k_full, (tile - 1) & 1, abort_flag, args.status);
      mbar_wait_warp(&sh.v_full, (tile - 1) & 1, abort_flag, args.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t idesc_qk = instr_desc(128, kBN, AB, false, false);
      constexpr uint32_t idesc_pv = instr_desc(128, D, AB, false, true);
      const uint32_t qa = smem_u32(q_tile), ka = smem_u32(k_tile), va = smem_u32(v_tile);
      bool ok = mbar_wait(&sh.q_full, 0, abort_flag, args.status);
      int issued = 0;  // PV commits issued
      for (int t = 0; ok; ++t) {
        const int slot = t % kRing;
        ok = mbar_wait(&sh.mask_full[slot], (t / kRing) & 1, abort_flag, args.status);
        if (!ok) break;
        const uint32_t fl = sh.flags[slot];
        mbar_arrive(&sh.mask_empty[slot]);
        if (fl & 2u) break;
        ok = mbar_wait(&sh.k_full, t & 1, abort_flag, args.status);
        if (ok && t > 0) ok = mbar_wait(&sh.pv_done, (t - 1) & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * 1024 + (kk & 3) * 32;
          const uint64_t adesc = smem_desc(qa + (kk >> 2) * L::kQPanel + (kk & 3) * 32, 16, 1024);
          const uint64_t bdesc = smem_desc(ka + koff, 16, L::kBoxBytes);
          umma_ss(tmem_s, adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sh.s_full);
        umma_commit(&sh.k_empty);
        ATTN_TRACE(2, 0x100u + t);
        ok = mbar_wait(&sh.p_full, t & 1, abort_flag, args.status);
        if (ok) ok = mbar_wait(&sh.v_full, t & 1, abort_flag, args.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bdesc = smem_desc(va + kk * 2 * L::kBoxBytes, 1024, L::kBoxBytes);
          umma_ts(tmem_o, tmem_s + kk * 8, bdesc, idesc_pv, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&sh.pv_done);
        umma_commit(&sh.v_empty);
        ATTN_TRACE(2, 0x200u + t);
        ++issued;
        if (fl & 1u) break;
      }
      // drain our MMAs before TMEM is released
      if (issued > 0) mbar_wait(&sh.pv_done, (issued - 1) & 1, abort_flag, args.status);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax
    const int quarter = warp & 3;                  // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;             // query row within the unit
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float m = -INFINITY, l = 0.0f;
    bool ok = true, empty = false;
    int t = 0;
    for (;; ++t) {
      const int slot = t % kRing;
      ok = mbar_wait_warp(&sh.mask_full[slot], (t / kRing) & 1, abort_flag, args.status);
      if (!ok) break;
      const uint32_t fl = sh.flags[slot];
      const uint32_t mw0 = sh.mask[slot][0], mw1 = sh.mask[slot][1], mw2 = sh.mask[slot][2], mw3 = sh.mask[slot][3];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.mask_empty[slot]);
      if (fl & 2u) {
        empty = true;
        break;
      }
      if (lane == 0) ATTN_TRACE(3 + quarter, 0x100u + t);
      ok = mbar_wait_warp(&sh.s_full, t & 1, abort_flag, args.status);
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) ATTN_TRACE(3 + quarter, 0x200u + t);
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32_sync(tmem_s + lane_off + c * 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[c * 32 + j] = __uint_as_float(v[j]);
      }
      const uint32_t mw[4] = {mw0, mw1, mw2, mw3};
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kBN; ++j) {
        const bool valid = (mw[j >> 5] >> (j & 31)) & 1u;
        s[j] = valid ? s[j] * args.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[j]);
      }
      // grow the running max lazily (only by > 8 in log2 units); rescaling O
      // is warp-collective because tcgen05.ld/st are .sync.aligned.  The
      // previous P.V is complete: this tile's QK^T was issued after it.
      const bool grow = (mx > m + 8.0f) || (m == -INFINITY && mx > -INFINITY);
      const bool rescale_me = grow && m != -INFINITY;
      if (__any_sync(0xffffffffu, rescale_me)) {
        const float f = rescale_me ? exp2f(m - mx) : 1.0f;
        l *= f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32_sync(tmem_o + lane_off + c * 32, v);
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            lo[j] = __float_as_uint(__uint_as_float(v[j]) * f);
            hi[j] = __float_as_uint(__uint_as_float(v[16 + j]) * f);
          }
          tmem_st16(tmem_o + lane_off + c * 32, lo);
          tmem_st16(tmem_o + lane_off + c * 32 + 16, hi);
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
        tmem_st16(tmem_s + lane_off + c * 16, part);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) ATTN_TRACE(3 + quarter, 0x300u + t);
      if (lane == 0) mbar_arrive(&sh.p_full);
      if (fl & 1u) break;
    }
    // epilogue
    const bool have_o = ok && !empty;
    if (have_o) ok = mbar_wait_warp(&sh.pv_done, t & 1, abort_flag, args.status);
    tc_fence_after();
    if (lane == 0) ATTN_TRACE(3 + quarter, 0x400u + (ok ? 1u : 0u));
    // TMEM reads are warp-collective; only the stores depend on the row
    using T = typename std::conditional<AB == 1, __nv_bfloat16, __half>::type;
    T* dst = nullptr;
    if (r < q_count && (ok || empty)) {
      const int prow = q_start + r;
      long long orow = prow;
      if (args.perm && prow < args.video) orow = args.perm[static_cast<long long>(head) * args.video + prow];
      if (orow < 0 || orow >= args.out_rows) record_status(args.status, kDevBadIndex);
      else dst = static_cast<T*>(args.out) + (static_cast<long long>(head) * args.out_rows + orow) * D;
    }
    __syncwarp();
    if (have_o && ok) {
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32_sync(tmem_o + lane_off + c * 32, v);
        if (dst) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a = __uint_as_float(v[j + 2 * e]) * inv, b = __uint_as_float(v[j + 2 * e + 1]) * inv;
              pw[e] = AB ? pack_bf16x2(a, b) : pack_f16x2(a, b);
            }
            reinterpret_cast<uint4*>(dst)[(c * 32 + j) / 8] = pk;
          }
        }
      }
    } else if (dst && empty) {
#pragma unroll
      for (int c = 0; c < D / 8; ++c) reinterpret_cast<uint4*>(dst)[c] = make_uint4(0, 0, 0, 0);
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
  if (threadIdx.x == 32) ATTN_TRACE(0, 4);
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

template <int D, int AB>
int launch_main(const void* q, const void* k, const void* v, const AttnArgs& a, int bh, int max_units,
                cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  if (!make_rows_map(&tq, q, static_cast<long long>(bh) * a.sq, D, kBM, AB) ||
      !make_rows_map(&tk, k, static_cast<long long>(bh) * a.sk, D, kBox, AB) ||
      !make_rows_map(&tv, v, static_cast<long long>(bh) * a.sk, D, kBox, AB))
    return kErrTensorMap;
  const int smem = Layout<D>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(sparse_attention_tc<D, AB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid(max_units, bh);
  sparse_attention_tc<D, AB><<<grid, kThreads, smem, stream>>>(tq, tk, tv, a);
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
  const size_t plan_smem = 2 * sizeof(int) * static_cast<size_t>(gq);
  if (plan_smem > 200 * 1024) return kErrUnsupported;
  if (plan_smem > 48 * 1024)
    cudaFuncSetAttribute(attn_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan_smem));
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return kErrInvalidValue;
  attn_plan_kernel<<<bh, 1024, plan_smem, stream>>>(q_sizes, k_sizes, ws, gq, gk, sq, sk, ws_stride);
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
  a.sq = sq;
  a.sk = sk;
  a.gq = gq;
  a.gk = gk;
  a.ws_stride = ws_stride;
  a.out_rows = sq;
  a.video = perm ? video : 0;
  a.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(d)));
  a.status = device_status_ptr();
  if (d == 128)
    return dtype ? launch_main<128, 1>(q, k, v, a, bh, static_cast<int>(max_units), stream)
                 : launch_main<128, 0>(q, k, v, a, bh, static_cast<int>(max_units), stream);
  return dtype ? launch_main<64, 1>(q, k, v, a, bh, static_cast<int>(max_units), stream)
               : launch_main<64, 0>(q, k, v, a, bh, static_cast<int>(max_units), stream);
}

// Workspace ints per head needed by launch_sparse_attention.
long long attention_ws_stride(int sq, int gq, int gk) {
  const long long max_units = (static_cast<long long>(sq) + kBM - 1) / kBM + gq;
  return 2 + gk + 3 * max_units;
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
