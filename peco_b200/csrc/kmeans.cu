// Lloyd k-means on sm_100a: nearest-centre assignment on the tensor core and
// a deterministic centroid update.
//
// Assignment (peco/kernels/kmeans.cu:139-175, peco/clustering.py:66-73):
//   label = argmin_c ||c||^2 - 2 x.c, lowest index on ties.
// The tokens of a PECO call are bf16, so x is exact as a bf16 MMA operand.
// Each fp32 centroid is split into two bf16 terms, c = c_hi + c_lo + r with
// |r| <= 2^-16 |c|, and S = X (C_hi + C_lo)^T is accumulated in fp32 in TMEM
// (tcgen05.mma, M=128 tokens, N<=256 centroids per chunk; both terms go into
// the same accumulator).  The computed distance is then within
//   E = 2^-12 ||x|| max||c|| + 2^-20 (max||c||^2 + 2 ||x|| max||c||)
// of the fp32 distance (split residual, fp32 accumulation and the final
// subtraction, with a 4x margin).  The epilogue finds the minimum, then every
// centroid within 2E of it: a single survivor is the fp32 argmin outright;
// several survivors (near-ties) are recomputed exactly in fp32 on the CUDA
// cores and the lowest index wins ties.  Labels therefore equal the fp32
// argmin except where two fp32 distances tie to rounding level.  fp32 inputs
// (the drop-in entry point) are split into bf16 hi + lo rows first (three MMA
// terms).
//
// The bf16 hi/lo centroid split is computed once per iteration -- by the
// update kernel, which produces the centroids -- and stored as the byte image
// the tensor core reads from shared memory, so an assignment CTA fetches it
// with bulk copies.  Token tiles arrive by TMA.  CTAs take equal-cost ranges
// of the (problem, head, tile) list.
//
// Update (peco/kernels/kmeans.cu:179-196, peco/clustering.py:74-80): tokens
// are stably sorted by label (counting sort), then one warp per cluster sums
// its tokens in ascending token order in fp32 -- the accumulation order of the
// reference's CPU scatter_add -- and divides by the count; empty clusters keep
// their previous centre.  No atomics: the result is deterministic and, for
// identical labels, bit-identical to the reference's CPU centroids.
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

// Fixed scratch of peco_recompute_cluster_centers_static: the stable sort's
// permutation (batch * tokens ints) followed by the cluster offsets
// (batch * (clusters + 1) ints).  One copy per device, 8 MiB.  Nothing in it
// needs to start at zero: every call writes the part it reads.
static __device__ __align__(256) int32_t g_update_scratch[1 << 21];

namespace peco {
namespace {

constexpr int kTileM = 128;
constexpr int kMaxCand = 4;
// warp 0: TMA / bulk-copy producer (and the centroid norms of each head);
// warp 1: MMA issuer and TMEM owner; warps 2-9: epilogue in two groups of
// four, group g taking the CTA's tiles of parity g in accumulator slot g.  A
// warp owns one TMEM lane quarter (32 tokens) and scans all of their centroid
// columns, so no warp waits for another's partial result and two tiles are
// scanned at once (a per-tile clock64 timeline of the earlier split -- two
// warps per row, half the columns each, merged through shared memory --
// showed the merge hand-off and its serial tail as the period's largest part)
constexpr int kEpiWarps = 8;
constexpr int kGroupWarps = 4;  // an epilogue group: one warp per TMEM lane quarter
constexpr int kMaxASlots = 4;          // token-tile ring depth when a CTA's centroid image leaves room
constexpr int kMmaWarp = 1, kEpiWarp0 = 2;
constexpr int kAssignThreads = 32 * (kEpiWarp0 + kEpiWarps);
// Near-tie tolerance of the tensor-core distance d' = |c|^2 - 2 x.(c_hi + c_lo)
// against the fp32 distance: |d' - d| <= kBoundScale |x| max|c| + kBoundTiny
// (max|c|^2 + 2 |x| max|c|).  The split residual is <= 2^-18 |x||c| and the
// largest accumulation error measured on B200 (1.3M tokens of the HV-480
// mixture, fp32 centres at four noise scales, compared with fp64) is
// 2^-18.2 |x| max|c|, so 2^-15 keeps a 9x margin over what was seen.  Any
// centre within twice the tolerance of the best is settled by an exact fp32
// recompute, so a label can only differ from the fp32 argmin at a tie.
constexpr float kBoundScale = 3.0517578125e-5f;    // 2^-15
constexpr float kBoundTiny = 9.5367431640625e-7f;  // 2^-20
constexpr int kCopyPiece = 32768;                  // bytes per bulk copy

__host__ __device__ constexpr int round16(int v) { return (v + 15) & ~15; }

// Centroid chunking: nc centroids per chunk (multiple of 16, <= 256).  The
// image of one (head, chunk) is b_bytes = 2 nc D 2 bytes: the hi term, then
// the lo term, each D/64 panels of nc rows x 128 bytes with the 128-byte
// swizzle (16-byte chunk q of row j at q ^ (j % 8)); rows past C are zero.
struct CenterGeom {
  int nc, nchunks, b_bytes, panel_bytes, term_bytes;
};
__host__ __device__ inline CenterGeom center_geom(int C, int D) {
  CenterGeom g;
  g.nc = round16(C < 256 ? C : 256);
  g.nchunks = (C + g.nc - 1) / g.nc;
  g.panel_bytes = g.nc * 128;
  g.term_bytes = g.nc * D * 2;
  g.b_bytes = 2 * g.term_bytes;
  return g;
}

// Byte offset of element d of centroid row j inside one chunk image term.
__device__ __forceinline__ int image_offset(const CenterGeom& g, int j, int d) {
  return (d >> 6) * g.panel_bytes + j * 128 + (((((d & 63) >> 3)) ^ (j & 7)) << 4) + (d & 7) * 2;
}

// Write E consecutive elements of centroid c (dims d0..d0+E-1, d0 % E == 0,
// E in {1, 2, 4}) as bf16 hi + lo into the image of one head.
template <int E>
__device__ __forceinline__ void write_image(unsigned char* img_head, const CenterGeom& g, int c, int d0,
                                            const float (&v)[E]) {
  unsigned char* chunk = img_head + static_cast<long long>(c / g.nc) * g.b_bytes;
  const int off = image_offset(g, c % g.nc, d0);
  __nv_bfloat16 hi[E], lo[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    hi[e] = __float2bfloat16_rn(v[e]);
    lo[e] = __float2bfloat16_rn(v[e] - __bfloat162float(hi[e]));
  }
  if constexpr (E == 4) {
    *reinterpret_cast<uint2*>(chunk + off) = *reinterpret_cast<const uint2*>(hi);
    *reinterpret_cast<uint2*>(chunk + g.term_bytes + off) = *reinterpret_cast<const uint2*>(lo);
  } else if constexpr (E == 2) {
    *reinterpret_cast<uint32_t*>(chunk + off) = *reinterpret_cast<const uint32_t*>(hi);
    *reinterpret_cast<uint32_t*>(chunk + g.term_bytes + off) = *reinterpret_cast<const uint32_t*>(lo);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      *reinterpret_cast<__nv_bfloat16*>(chunk + image_offset(g, c % g.nc, d0 + e)) = hi[e];
      *reinterpret_cast<__nv_bfloat16*>(chunk + g.term_bytes + image_offset(g, c % g.nc, d0 + e)) = lo[e];
    }
  }
}

// Norms and image of a set of centroids: one warp per padded centroid row
// (rows past C get a zero image).  centers [B, C, D]; norms [B, C];
// image [B, nchunks * b_bytes].
struct PrepJob {
  const float* centers;
  float* norms;
  unsigned char* image;
  int C;
};
struct PrepJobs {
  PrepJob job[2];   // blockIdx.y selects the job (the Q and K centres of one fit)
};
template <int D>
__global__ void center_prep_kernel(const PrepJobs jobs, int bh) {
  constexpr int E = D / 32;
  const PrepJob J = blockIdx.y ? jobs.job[1] : jobs.job[0];  // no dynamic index into the parameters
  const int C = J.C;
  const CenterGeom g = center_geom(C, D);
  const int padded = g.nchunks * g.nc;
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(bh) * padded) return;
  const int head = static_cast<int>(w / padded), c = static_cast<int>(w % padded);
  float v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = c < C ? J.centers[(static_cast<long long>(head) * C + c) * D + lane * E + e] : 0.0f;
  if (J.image) write_image<E>(J.image + static_cast<long long>(head) * g.nchunks * g.b_bytes, g, c, lane * E, v);
  if (c < C && J.norms) {
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) s = fmaf(v[e], v[e], s);
    s = warp_sum(s);
    if (lane == 0) J.norms[static_cast<long long>(head) * C + c] = s;
  }
}

// fp32 rows -> bf16 hi and lo rows (hi = rn(x), lo = rn(x - hi))
__global__ void split_rows_kernel(const float4* __restrict__ x, uint2* __restrict__ hi, uint2* __restrict__ lo,
                                  long long n4) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 f = x[i];
    const float v[4] = {f.x, f.y, f.z, f.w};
    __nv_bfloat16 h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = __float2bfloat16_rn(v[e]);
      l[e] = __float2bfloat16_rn(v[e] - __bfloat162float(h[e]));
    }
    hi[i] = *reinterpret_cast<const uint2*>(h);
    lo[i] = *reinterpret_cast<const uint2*>(l);
  }
}

struct AssignJob {
  int tokens, clusters;
  long long head_rows;          // rows between consecutive heads in the token maps
  const float* x32;             // fp32 rows for the exact recompute (split mode), else null
  const __nv_bfloat16* xb;      // bf16 rows for the exact recompute (bf16 mode), else null
  const float* centers;         // [B, C, D] fp32 (exact recompute of near-ties)
  const float* norms;           // [B, C]
  const unsigned char* image;   // [B, nchunks * b_bytes]
  int32_t* labels;              // [B, tokens]
  const float* xn_in;           // optional [B, tokens] token norms |x| (skips recomputing them)
  float* xn_out;                // optional [B, tokens]: |x| written for later iterations
};

struct AssignJobs {
  AssignJob job[2];
  int njobs, bh;
  long long items[2];   // (head, tile) items per problem
  long long cost[2];    // cost of one item (centroid columns)
  int ncta;
  // split[j] > 0: each (problem j, head) group is cut into split[j] CTAs of
  // consecutive tiles, so no CTA changes centroid sets mid-launch; 0: CTAs
  // take equal-cost ranges of the flattened item list
  int split[2];
  int dyn_smem;  // dynamic shared memory of the launch (bytes)
};

struct AssignMaps {
  CUtensorMap xhi[2], xlo[2];   // bf16 token rows (lo: split mode only), box 64 x 128
};

struct __align__(8) AssignBars {
  uint64_t g_full, g_free;
  uint64_t a_full[kMaxASlots], a_empty[kMaxASlots];
  uint64_t b_full[2], b_empty[2];
  uint64_t acc_full[2], acc_empty[2];  // per accumulator slot = per epilogue group
  uint32_t tmem_base;
  int abort_flag;
};

// Shared-memory carve-up common to every problem of a launch.
struct AssignSmem {
  int resident;     // 1: each head's single chunk stays in smem; 0: chunks stream through 2 slots
  int nbslots, naslots;
  int b_bytes, a_bytes, a_off, cn_off, cn_cap, smem;
};
__host__ __device__ inline AssignSmem assign_smem(int C0, int C1, int njobs, int D, bool split) {
  AssignSmem s;
  int bmax = 0, cmax = 0;
  bool all_single = true;
  for (int j = 0; j < njobs; ++j) {
    const CenterGeom g = center_geom(j ? C1 : C0, D);
    bmax = bmax > g.b_bytes ? bmax : g.b_bytes;
    const int cpad = (g.nchunks * g.nc + 31) & ~31;  // whole 32-column blocks
    cmax = cmax > cpad ? cmax : cpad;
    all_single = all_single && g.nchunks == 1;
  }
  s.resident = all_single ? 1 : 0;
  s.nbslots = all_single ? 1 : 2;
  s.b_bytes = bmax;
  s.a_bytes = kTileM * D * 2 * (split ? 2 : 1);
  s.cn_cap = cmax;
  s.naslots = 2;
  for (;;) {
    s.a_off = s.nbslots * s.b_bytes;
    s.cn_off = s.a_off + s.naslots * s.a_bytes;
      s.smem = 1024 + s.cn_off + ((cmax * 4 + 1023) & ~1023);
    if (s.smem <= 227 * 1024) break;
    if (s.nbslots > 1) s.nbslots = 1;       // streamed chunks: single-buffered
    else if (s.naslots > 1) s.naslots = 1;  // then a single token tile
    else break;
  }
  return s;
}

// item f of the flattened list: problem j, head, tile (head-major per problem)
struct Item {
  int j, head, tile;
};
__device__ __forceinline__ Item decode_item(const AssignJobs& a, long long f) {
  Item it;
  it.j = f < a.items[0] ? 0 : 1;
  const long long local = it.j ? f - a.items[0] : f;
  const int nt = (a.job[it.j].tokens + kTileM - 1) / kTileM;
  it.head = static_cast<int>(local / nt);
  it.tile = static_cast<int>(local % nt);
  return it;
}
// The items of a CTA are consecutive: decode the first once, then step
// (tile, head, problem) without 64-bit divisions in the per-item loops.
struct ItemCursor {
  Item it;
  int nt;  // tiles per head of the current problem
  __device__ __forceinline__ void start(const AssignJobs& a, long long f) {
    it = decode_item(a, f);
    nt = (a.job[it.j].tokens + kTileM - 1) / kTileM;
  }
  __device__ __forceinline__ bool last_in_group() const { return it.tile + 1 == nt; }
  __device__ __forceinline__ void next(const AssignJobs& a) {
    if (++it.tile == nt) {
      it.tile = 0;
      if (++it.head == a.bh) {
        it.head = 0;
        ++it.j;
        nt = (a.job[it.j & 1].tokens + kTileM - 1) / kTileM;
      }
    }
  }
};
// position in a ring of n slots: slot s in its round's phase parity p
struct Ring {
  int s = 0, n = 1;
  uint32_t p = 0;
  __device__ __forceinline__ void next() {
    if (++s == n) {
      s = 0;
      p ^= 1u;
    }
  }
};

// first item whose cumulative cost reaches x
__device__ __forceinline__ long long item_at(const AssignJobs& a, long long x) {
  const long long c0 = a.items[0] * a.cost[0];
  if (x <= c0) return (x + a.cost[0] - 1) / a.cost[0];
  const long long f = a.items[0] + (x - c0 + a.cost[1] - 1) / a.cost[1];
  const long long total = a.items[0] + (a.njobs > 1 ? a.items[1] : 0);
  return f < total ? f : total;
}

template <int D, bool SPLIT>
__global__ void __launch_bounds__(kAssignThreads, 1) kmeans_assign_kernel(const __grid_constant__ AssignMaps maps,
                                                                        const AssignJobs jobs, unsigned* status) {
  long long f_begin, f_end;
  if (jobs.split[0] > 0) {
    const int b = static_cast<int>(blockIdx.x);
    const int j = b < jobs.bh * jobs.split[0] ? 0 : 1;
    const int local = j ? b - jobs.bh * jobs.split[0] : b;
    const int head = local / jobs.split[j], piece = local % jobs.split[j];
    const long long nt = (jobs.job[j].tokens + kTileM - 1) / kTileM;
    const long long first = (j ? jobs.items[0] : 0) + head * nt;
    f_begin = first + nt * piece / jobs.split[j];
    f_end = first + nt * (piece + 1) / jobs.split[j];
  } else {
    const long long total_cost = jobs.items[0] * jobs.cost[0] + (jobs.njobs > 1 ? jobs.items[1] * jobs.cost[1] : 0);
    f_begin = item_at(jobs, total_cost * blockIdx.x / jobs.ncta);
    f_end = item_at(jobs, total_cost * (blockIdx.x + 1) / jobs.ncta);
  }
  if (f_begin >= f_end) return;
  const AssignSmem S = assign_smem(jobs.job[0].clusters, jobs.njobs > 1 ? jobs.job[1].clusters : 1, jobs.njobs, D, SPLIT);
  // The token tile in shared memory is read by the MMA, and by its epilogue
  // group only to compute |x| (when no cached norms are given): the exact
  // recompute of near-ties reads its rows from global memory, so a slot is
  // free for the next tile as soon as the MMAs (and the |x| pass, if any) are
  // done.
  const bool epi_reads_a = jobs.job[0].xn_in == nullptr || (jobs.njobs > 1 && jobs.job[1].xn_in == nullptr);

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1 KB-aligned base, derived from smem_raw by pointer arithmetic so that
  // the compiler keeps shared-memory (not generic) accesses through it
  unsigned char* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  // Token-tile ring: a CTA that serves one resident group takes every slot its
  // own image leaves free (up to kMaxASlots), the norms sit at the end.
  int a_off = S.a_off, cn_off = S.cn_off, NA = S.naslots;
  if (jobs.split[0] > 0 && S.resident) {
    const Item first = decode_item(jobs, f_begin);
    a_off = center_geom(jobs.job[first.j].clusters, D).b_bytes;
    cn_off = (jobs.dyn_smem - 1024 - S.cn_cap * 4) & ~1023;
    const int fit = (cn_off - a_off) / S.a_bytes;
    NA = fit < kMaxASlots ? fit : kMaxASlots;
    if (NA < S.naslots) {  // never fewer than the launch-wide layout
      a_off = S.a_off;
      cn_off = S.cn_off;
      NA = S.naslots;
    }
  }
  float* cn = reinterpret_cast<float*>(base + cn_off);  // centroid norms of the current head (+inf past C)
  __shared__ AssignBars sb;
  volatile int* abort_flag = &sb.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&sb.g_full, 32);
    mbar_init(&sb.g_free, 1 + kEpiWarps);
    for (int i = 0; i < NA; ++i) {
      mbar_init(&sb.a_full[i], 1);
      // the tile's MMAs always release it; its epilogue group too when it
      // reads the tile for the token norms
      mbar_init(&sb.a_empty[i], 1 + (epi_reads_a ? kGroupWarps : 0));
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sb.b_full[i], 1);
      mbar_init(&sb.b_empty[i], 1);
      mbar_init(&sb.acc_full[i], 1);
      mbar_init(&sb.acc_empty[i], kGroupWarps);
    }
    sb.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sb.tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;
  const int a_panel = kTileM * 128;  // bytes per 64-column panel of an A tile
  // group = (problem, head): the centroids in smem change with it
  auto group_of = [&](const Item& it) { return it.j * jobs.bh + it.head; };
  // Tiles go in pairs of consecutive items of one group (a single tile where
  // the group or the range ends): the two tiles' MMAs alternate chunk by
  // chunk, so each streamed centroid chunk serves both.  Every role derives
  // the same pairing from its own cursor.
  auto pair_size = [&](long long f, const ItemCursor& cur) { return (f + 1 < f_end && !cur.last_in_group()) ? 2 : 1; };

  if (warp == 0) {
    // ------------------------------------------------ TMA / bulk producer
    if (lane == 0) {
      prefetch_tensormap(&maps.xhi[0]);
      if (jobs.njobs > 1) prefetch_tensormap(&maps.xhi[1]);
    }
    bool ok = true;
    int group = -1, ngroups = 0, bchunk = 0;
    int i = 0;
    ItemCursor cur;
    cur.start(jobs, f_begin);
    Ring ring;
    ring.n = NA;
    for (long long f = f_begin; f < f_end && ok;) {
      const int np = pair_size(f, cur);
      const Item it0 = cur.it;
      const AssignJob& J = jobs.job[it0.j];
      const CenterGeom cg = center_geom(J.clusters, D);
      const unsigned char* img = J.image + static_cast<long long>(it0.head) * cg.nchunks * cg.b_bytes;
      if (group_of(it0) != group) {
        if (ngroups > 0) ok = mbar_wait_warp(&sb.g_free, (ngroups - 1) & 1, abort_flag, status);
        if (!ok) break;
        // centroid norms (+inf for padding columns) and, when resident, the image
        const float* nr = J.norms + static_cast<long long>(it0.head) * J.clusters;
        for (int c = lane; c < ((cg.nchunks * cg.nc + 31) & ~31); c += 32) cn[c] = c < J.clusters ? nr[c] : INFINITY;
        if (lane == 0) {
          mbar_arrive_expect_tx(&sb.g_full, S.resident ? cg.b_bytes : 0);
          if (S.resident)
            for (int off = 0; off < cg.b_bytes; off += kCopyPiece)
              bulk_load(base + off, img + off, min(kCopyPiece, cg.b_bytes - off), &sb.g_full);
        } else {
          mbar_arrive(&sb.g_full);
        }
        group = group_of(it0);
        ++ngroups;
      }
      for (int p = 0; p < np && ok; ++p, ++f, ++i, cur.next(jobs), ring.next()) {
        const Item it = cur.it;
        const int s = ring.s;
        if (i >= NA) ok = mbar_wait_warp(&sb.a_empty[s], ring.p ^ 1u, abort_flag, status);
        if (!ok) break;
        if (lane == 0) {
          unsigned char* a = base + a_off + s * S.a_bytes;
          mbar_arrive_expect_tx(&sb.a_full[s], S.a_bytes);
          const int row = static_cast<int>(static_cast<long long>(it.head) * J.head_rows + static_cast<long long>(it.tile) * kTileM);
#pragma unroll
          for (int q = 0; q < D / 64; ++q) {
            tma_load_2d(a + q * a_panel, &maps.xhi[it.j], 64 * q, row, &sb.a_full[s]);
            if (SPLIT) tma_load_2d(a + kTileM * D * 2 + q * a_panel, &maps.xlo[it.j], 64 * q, row, &sb.a_full[s]);
          }
        }
        __syncwarp();
      }
      if (!S.resident) {
        // each chunk once per pair
        for (int k = 0; k < cg.nchunks && ok; ++k, ++bchunk) {
          const int bs = bchunk % S.nbslots, bu = bchunk / S.nbslots;
          if (bu > 0) ok = mbar_wait_warp(&sb.b_empty[bs], (bu - 1) & 1, abort_flag, status);
          if (!ok) break;
          if (lane == 0) {
            mbar_arrive_expect_tx(&sb.b_full[bs], cg.b_bytes);
            for (int off = 0; off < cg.b_bytes; off += kCopyPiece)
              bulk_load(base + bs * S.b_bytes + off, img + static_cast<long long>(k) * cg.b_bytes + off,
                        min(kCopyPiece, cg.b_bytes - off), &sb.b_full[bs]);
          }
          __syncwarp();
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      bool ok = true;
      int group = -1, ngroups = 0, bchunk = 0;
      int uses0 = 0, uses1 = 0;  // accumulator slot uses so far
      int i = 0;
      ItemCursor cur;
      cur.start(jobs, f_begin);
      Ring ring;
      ring.n = NA;
      for (long long f = f_begin; f < f_end && ok;) {
        const int np = pair_size(f, cur);
        const Item it0 = cur.it;
        const CenterGeom cg = center_geom(jobs.job[it0.j].clusters, D);
        const uint32_t idesc = instr_desc(128, cg.nc, 1, false, false);
        if (group_of(it0) != group) {
          ok = mbar_wait(&sb.g_full, ngroups & 1, abort_flag, status);
          group = group_of(it0);
          ++ngroups;
        }
        // the pair's ring slots and accumulator slots (slot = tile index parity)
        int as_of[2] = {i & 1, (i + 1) & 1};
        int rs_of[2] = {ring.s, 0};
        uint32_t rp_of[2] = {ring.p, 0};
        bool last_of[2] = {np == 1 && cur.last_in_group(), false};
        {
          Ring r2 = ring;
          ItemCursor c2 = cur;
          r2.next();
          c2.next(jobs);
          rs_of[1] = r2.s;
          rp_of[1] = r2.p;
          if (np == 2) last_of[1] = f + 2 >= f_end || c2.last_in_group();
        }
        if (np == 1) last_of[0] = last_of[0] || f + 1 >= f_end;
#pragma unroll
        for (int p = 0; p < 2; ++p)
          if (p < np && ok) ok = mbar_wait(&sb.a_full[rs_of[p]], rp_of[p], abort_flag, status);
        for (int k = 0; k < cg.nchunks && ok; ++k) {
          int bs = 0;
          if (!S.resident) {
            bs = bchunk % S.nbslots;
            ok = mbar_wait(&sb.b_full[bs], (bchunk / S.nbslots) & 1, abort_flag, status);
            ++bchunk;
          }
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            if (p >= np || !ok) continue;
            const int as = as_of[p];
            const int u = as ? uses1 : uses0;
            if (u > 0) ok = mbar_wait(&sb.acc_empty[as], (u - 1) & 1, abort_flag, status);
            if (!ok) continue;
            if (as) ++uses1;
            else ++uses0;
            tc_fence_after();
            const uint32_t a_hi = smem_u32(base + a_off + rs_of[p] * S.a_bytes);
            const uint32_t a_lo = a_hi + kTileM * D * 2;
            const uint32_t b_hi = smem_u32(base + bs * S.b_bytes);
            const uint32_t b_lo = b_hi + cg.term_bytes;
            const uint32_t acc = tmem + as * 256;
            // terms, smallest first: x.c_lo, [x_lo.c_hi], x.c_hi
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off_a = (kk >> 2) * a_panel + (kk & 3) * 32;
              const uint32_t off_b = (kk >> 2) * cg.panel_bytes + (kk & 3) * 32;
              umma_ss(acc, smem_desc(a_hi + off_a, 16, 1024), smem_desc(b_lo + off_b, 16, 1024), idesc, kk > 0 ? 1u : 0u);
            }
            if (SPLIT) {
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t off_a = (kk >> 2) * a_panel + (kk & 3) * 32;
                const uint32_t off_b = (kk >> 2) * cg.panel_bytes + (kk & 3) * 32;
                umma_ss(acc, smem_desc(a_lo + off_a, 16, 1024), smem_desc(b_hi + off_b, 16, 1024), idesc, 1u);
              }
            }
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off_a = (kk >> 2) * a_panel + (kk & 3) * 32;
              const uint32_t off_b = (kk >> 2) * cg.panel_bytes + (kk & 3) * 32;
              umma_ss(acc, smem_desc(a_hi + off_a, 16, 1024), smem_desc(b_hi + off_b, 16, 1024), idesc, 1u);
            }
            umma_commit(&sb.acc_full[as]);
            if (k + 1 == cg.nchunks) {
              umma_commit(&sb.a_empty[rs_of[p]]);
              if (last_of[p]) umma_commit(&sb.g_free);
            }
          }
          if (ok && !S.resident) umma_commit(&sb.b_empty[bs]);
        }
        for (int p = 0; p < np; ++p, ++f, ++i, cur.next(jobs), ring.next()) {
        }
      }
      // drain our MMAs before TMEM is released
      if (uses0 > 0) mbar_wait(&sb.acc_full[0], (uses0 - 1) & 1, abort_flag, status);
      if (uses1 > 0) mbar_wait(&sb.acc_full[1], (uses1 - 1) & 1, abort_flag, status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- epilogue
    // Group g = (warp - 2) / 4 takes the CTA's tiles of parity g: each of its
    // warps owns one TMEM lane quarter (32 tokens) and scans every centroid
    // column of its rows, so a tile needs no exchange between warps and the
    // two groups work on two tiles at once.
    const int quarter = warp & 3;
    const int eg = (warp - kEpiWarp0) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    int group = -1, ngroups = 0, use = 0;
    float cmax = 0.0f;
    int i = 0;
    ItemCursor cur;
    cur.start(jobs, f_begin);
    Ring ring;
    ring.n = NA;
    for (long long f = f_begin; f < f_end && ok; ++f, ++i, cur.next(jobs), ring.next()) {
      const Item it = cur.it;
      const AssignJob& J = jobs.job[it.j];
      const int C = J.clusters;
      const CenterGeom cg = center_geom(C, D);
      if (group_of(it) != group) {
        ok = mbar_wait_warp(&sb.g_full, ngroups & 1, abort_flag, status);
        if (!ok) break;
        float m = 0.0f;
        for (int c = lane; c < C; c += 32) m = fmaxf(m, cn[c]);
        cmax = sqrtf(warp_max(m));
        group = group_of(it);
        ++ngroups;
      }
      const bool last_in_group = f + 1 >= f_end || cur.last_in_group();
      if ((i & 1) != eg) {
        // the other group's tile; this warp's tiles of the group are done
        if (last_in_group && lane == 0) mbar_arrive(&sb.g_free);
        __syncwarp();
        continue;
      }
      const int s = ring.s;
      // Only a launch whose epilogue reads the tile waits for it (and holds
      // the slot until it has): otherwise the MMA may already have released
      // the slot and the producer refilled it, so this phase parity would
      // name a later tile.  acc_full below orders everything else.
      if (epi_reads_a) ok = mbar_wait_warp(&sb.a_full[s], ring.p, abort_flag, status);
      if (!ok) break;
      const unsigned char* a_hi = base + a_off + s * S.a_bytes;
      // the token norm: cached by an earlier iteration, or computed here
      const int tok_r = it.tile * kTileM + r;
      const bool cached_xn = J.xn_in != nullptr;
      float xn = 0.0f;
      if (cached_xn) {
        if (tok_r < J.tokens) xn = J.xn_in[static_cast<long long>(it.head) * J.tokens + tok_r];
      } else {
        float ss = 0.0f;
#pragma unroll 1
        for (int ch = 0; ch < D / 8; ++ch) {
          const int off = (ch >> 3) * a_panel + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
          const uint4 u = *reinterpret_cast<const uint4*>(a_hi + off);
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
          float2 lo2[4] = {};
          if (SPLIT) {
            const uint4 w = *reinterpret_cast<const uint4*>(a_hi + kTileM * D * 2 + off);
            const __nv_bfloat162* l2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) lo2[e] = __bfloat1622float2(l2[e]);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f2 = __bfloat1622float2(h2[e]);
            const float x0 = f2.x + lo2[e].x, x1 = f2.y + lo2[e].y;
            ss = fmaf(x0, x0, ss);
            ss = fmaf(x1, x1, ss);
          }
        }
        xn = sqrtf(ss);
        if (J.xn_out && tok_r < J.tokens) J.xn_out[static_cast<long long>(it.head) * J.tokens + tok_r] = xn;
      }
      if (epi_reads_a) {  // done with the tile in shared memory
        __syncwarp();
        if (lane == 0) mbar_arrive(&sb.a_empty[s]);
      }
      const float E2 = 2.0f * (kBoundScale * xn * cmax + kBoundTiny * (cmax * cmax + 2.0f * xn * cmax));
      float best = INFINITY;
      float cd[kMaxCand];
      int ci[kMaxCand];
      int ncand = 0;
      bool overflow = false;
      // keep entries within ``t`` (order preserved)
      auto prune = [&](float t) {
        int m = 0;
#pragma unroll
        for (int q = 0; q < kMaxCand; ++q) {
          const bool keep = q < ncand && cd[q] <= t;
#pragma unroll
          for (int p = 0; p < kMaxCand; ++p)
            if (keep && p == m) {
              cd[p] = cd[q];
              ci[p] = ci[q];
            }
          m += keep ? 1 : 0;
        }
        ncand = m;
      };
      auto push = [&](float dj, int c) {
        if (ncand < kMaxCand) {
#pragma unroll
          for (int q = 0; q < kMaxCand; ++q)
            if (q == ncand) {
              cd[q] = dj;
              ci[q] = c;
            }
          ++ncand;
        } else {
          overflow = true;
        }
      };
      for (int k = 0; k < cg.nchunks && ok; ++k, ++use) {
        ok = mbar_wait_warp(&sb.acc_full[eg], use & 1, abort_flag, status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + eg * 256 + lane_off;
        const float* cnk = cn + k * cg.nc;
        const int nblk = cg.nc / 32 + ((cg.nc & 31) ? 1 : 0);
        // Two passes over the chunk's columns, each value's distance
        // d = |c|^2 - 2 x.c recomputed identically (one paired FMA per two
        // columns).  Pass 1: the chunk's best distance (independent min
        // chains).  Pass 2: how many columns lie within the near-tie
        // threshold of the running best and, from that count and a weighted
        // sum of their column numbers, the column itself when it is alone.
        // Both passes are mostly min / compare / FMA-pipe adds: the compare-
        // select argmin with a tracked runner-up they replace spent about
        // five half-rate ALU instructions per value, which bounded the kernel.
        // The block loops stay rolled: the unrolled body must fit the
        // instruction cache.
        auto dist2 = [&](const uint32_t* v, const float4* c4, int q, float2& lo, float2& hi) {
          const float4 nq = c4[q];
          const float2 m2 = make_float2(-2.0f, -2.0f);
          lo = ffma2(make_float2(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1])), m2, make_float2(nq.x, nq.y));
          hi = ffma2(make_float2(__uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])), m2, make_float2(nq.z, nq.w));
        };
        float mins[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mins[e] = INFINITY;
#pragma unroll 1
        for (int b = 0; b < nblk; ++b) {
          uint32_t v[32];
          tmem_ld32_sync(acc + b * 32, v);
          const float4* c4 = reinterpret_cast<const float4*>(cnk + b * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float2 lo, hi;
            dist2(v, c4, q, lo, hi);
            mins[q] = fminf(mins[q], fminf(fminf(lo.x, lo.y), fminf(hi.x, hi.y)));
          }
        }
        float m1 = fminf(fminf(fminf(mins[0], mins[1]), fminf(mins[2], mins[3])),
                         fminf(fminf(mins[4], mins[5]), fminf(mins[6], mins[7])));
        best = fminf(best, m1);
        const float thr = best + E2;
        if (ncand > 0) prune(thr);
        float count = 0.0f, where = 0.0f;
        if (__any_sync(0xffffffffu, m1 <= thr)) {
#pragma unroll 1
          for (int b = 0; b < nblk; ++b) {
            uint32_t v[32];
            tmem_ld32_sync(acc + b * 32, v);
            const float4* c4 = reinterpret_cast<const float4*>(cnk + b * 32);
            float2 cnt2 = make_float2(0.0f, 0.0f), pos2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float2 lo, hi;
              dist2(v, c4, q, lo, hi);
              const float2 f_lo = make_float2(lo.x <= thr ? 1.0f : 0.0f, lo.y <= thr ? 1.0f : 0.0f);
              const float2 f_hi = make_float2(hi.x <= thr ? 1.0f : 0.0f, hi.y <= thr ? 1.0f : 0.0f);
              cnt2 = fadd2(cnt2, fadd2(f_lo, f_hi));
              pos2 = ffma2(f_lo, make_float2(4 * q, 4 * q + 1), pos2);
              pos2 = ffma2(f_hi, make_float2(4 * q + 2, 4 * q + 3), pos2);
            }
            const float cnt_b = cnt2.x + cnt2.y;
            count += cnt_b;
            where += fmaf(cnt_b, static_cast<float>(k * cg.nc + b * 32), pos2.x + pos2.y);
          }
        }
        // candidates of this chunk: none (m1 > thr), exactly its best (one
        // column within the threshold), or several -- then rescan it (rare)
        const bool many = count > 1.5f;
        const int i1 = static_cast<int>(where);
        if (count > 0.5f && !many) push(m1, i1);
        if (__any_sync(0xffffffffu, many)) {
#pragma unroll 1
          for (int b = 0; b < nblk; ++b) {
            uint32_t v[32];
            tmem_ld32_sync(acc + b * 32, v);
            const float4* c4 = reinterpret_cast<const float4*>(cnk + b * 32);
            unsigned m = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 nq = c4[q];
              m |= (fmaf(-2.0f, __uint_as_float(v[4 * q + 0]), nq.x) <= thr ? 1u : 0u) << (4 * q + 0);
              m |= (fmaf(-2.0f, __uint_as_float(v[4 * q + 1]), nq.y) <= thr ? 1u : 0u) << (4 * q + 1);
              m |= (fmaf(-2.0f, __uint_as_float(v[4 * q + 2]), nq.z) <= thr ? 1u : 0u) << (4 * q + 2);
              m |= (fmaf(-2.0f, __uint_as_float(v[4 * q + 3]), nq.w) <= thr ? 1u : 0u) << (4 * q + 3);
            }
            if (!many) m = 0;
            // distances recorded as the chunk's best (a lower bound): a later
            // prune keeps them and the exact recompute settles them
            while (m) {
              const int jb = __ffs(m) - 1;
              m &= m - 1;
              push(m1, k * cg.nc + b * 32 + jb);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sb.acc_empty[eg]);
      }
      if (!ok) break;
      {
        const int tok = it.tile * kTileM + r;
        const bool valid = tok < J.tokens;
        if (ncand > 1) prune(best + E2);
        int label = ncand > 0 ? ci[0] : 0;
        // Near-ties are recomputed in exact fp32, one token at a time by the
        // whole warp: lane l owns D/32 consecutive dimensions, so each
        // candidate centroid row is one coalesced load, and all candidates of
        // the token are in flight together.
        unsigned amb = __ballot_sync(0xffffffffu, valid && (overflow || ncand > 1));
        constexpr int E = D / 32;
        const float* cen = J.centers + static_cast<long long>(it.head) * C * D;
        while (amb) {
          const int src = __ffs(amb) - 1;
          amb &= amb - 1;
          const int stok = __shfl_sync(0xffffffffu, tok, src);
          const int n = __shfl_sync(0xffffffffu, overflow ? -1 : ncand, src);
          float xv[E];
          if (SPLIT) {
            const float* xr = J.x32 + (static_cast<long long>(it.head) * J.head_rows + stok) * D + lane * E;
#pragma unroll
            for (int e = 0; e < E; ++e) xv[e] = xr[e];
          } else {
            // the token row from global memory (its shared-memory tile may already hold the next tile)
            const __nv_bfloat16* xr = J.xb + (static_cast<long long>(it.head) * J.head_rows + stok) * D + lane * E;
#pragma unroll
            for (int e = 0; e < E; ++e) xv[e] = __bfloat162float(xr[e]);
          }
          float bd = INFINITY;
          int bl = 0x7fffffff;
          auto score = [&](int id, float partial) {
            const float dot = warp_sum(partial);
            const float e = __fsub_rn(cn[id], 2.0f * dot);
            if (e < bd || (e == bd && id < bl)) {
              bd = e;
              bl = id;
            }
          };
          if (n >= 0) {
            float part[kMaxCand];
            int ids[kMaxCand];
#pragma unroll
            for (int q = 0; q < kMaxCand; ++q) {
              ids[q] = __shfl_sync(0xffffffffu, ci[q], src);
              part[q] = 0.0f;
              if (q < n) {
                const float* cr = cen + static_cast<long long>(ids[q]) * D + lane * E;
#pragma unroll
                for (int e = 0; e < E; ++e) part[q] = fmaf(xv[e], cr[e], part[q]);
              }
            }
#pragma unroll
            for (int q = 0; q < kMaxCand; ++q)
              if (q < n) score(ids[q], part[q]);
          } else {
#pragma unroll 1
            for (int c0 = 0; c0 < C; c0 += 4) {
              float part[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                part[q] = 0.0f;
                const int id = min(c0 + q, C - 1);
                const float* cr = cen + static_cast<long long>(id) * D + lane * E;
#pragma unroll
                for (int e = 0; e < E; ++e) part[q] = fmaf(xv[e], cr[e], part[q]);
              }
#pragma unroll
              for (int q = 0; q < 4; ++q)
                if (c0 + q < C) score(c0 + q, part[q]);
            }
          }
          if (lane == src) label = bl;
        }
        if (valid) J.labels[static_cast<long long>(it.head) * J.tokens + tok] = label;
      }
      __syncwarp();
      if (lane == 0 && last_in_group) mbar_arrive(&sb.g_free);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Centroid update, one warp per cluster.  x rows of head b are
// x + (b * head_rows + t) * D.  Also writes ||mean||^2 for the next assignment.
struct UpdateJob {
  const void* x;
  long long head_rows;
  int tokens;
  int clusters;
  const int32_t* perm;      // [B, tokens] stable sort by label
  const int32_t* offsets;   // [B, C+1]
  const float* previous;    // [B, C, D]
  float* means;             // [B, C, D]
  float* sums;              // optional [B, C, D]
  float* norms;             // optional [B, C]
  unsigned char* image;     // optional [B, nchunks * b_bytes]: bf16 hi/lo image of the means
  int big_rows;             // > 0: clusters above this many rows are left to kmeans_update_big_kernel
};
struct UpdateJobs {
  UpdateJob job[2];
};

// E consecutive elements of a row as fp32, in one vector load when possible.
template <typename T, int E>
__device__ __forceinline__ void load_lane_elems(const T* row, float (&v)[E]) {
  if constexpr (sizeof(T) == 2 && E == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(row);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = to_f32<T>(h[e]);
  } else if constexpr (sizeof(T) == 4 && E == 4) {
    const float4 f = *reinterpret_cast<const float4*>(row);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = to_f32<T>(row[e]);
  }
}

// A lane's E consecutive elements of a row, kept as raw words until summed.
template <typename T, int E>
struct LaneRaw {
  static constexpr int kBytes = E * static_cast<int>(sizeof(T));
  static constexpr int kWords = (kBytes + 3) / 4;
  uint32_t w[kWords];
  __device__ __forceinline__ void load(const T* row) {
    if constexpr (kBytes == 16) {
      const uint4 u = *reinterpret_cast<const uint4*>(row);
      w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
    } else if constexpr (kBytes == 8) {
      const uint2 u = *reinterpret_cast<const uint2*>(row);
      w[0] = u.x; w[1] = u.y;
    } else if constexpr (kBytes == 4) {
      w[0] = *reinterpret_cast<const uint32_t*>(row);
    } else {
      T* h = reinterpret_cast<T*>(w);
#pragma unroll
      for (int e = 0; e < E; ++e) h[e] = row[e];
    }
  }
  __device__ __forceinline__ float get(int e) const { return to_f32<T>(reinterpret_cast<const T*>(w)[e]); }
};

// One warp per cluster, two warps per block (a block slot frees as soon as its
// two clusters are done, so uneven cluster sizes hold few warps back); lane l
// owns elements [l*E, (l+1)*E).  The cluster's token ids arrive 32 at a time
// in one coalesced load (the next batch is prefetched), 16 rows are in flight
// at once, and the sums run strictly in ascending token order (bit-exact with
// a sequential scatter-add).
constexpr int kUpdateThreads = 64;
template <int D, typename T>
__global__ void __launch_bounds__(kUpdateThreads, 8) kmeans_update_kernel(const UpdateJobs jobs, int bh, unsigned* status) {
  const UpdateJob& J = jobs.job[blockIdx.y];
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(bh) * J.clusters) return;
  const int head = static_cast<int>(w / J.clusters);
  const int c = static_cast<int>(w - static_cast<long long>(head) * J.clusters);
  constexpr int E = D / 32;                            // elements per lane
  constexpr int kRows = 16;                            // rows in flight
  const int start = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c];
  int end = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c + 1];
  const int32_t* perm = J.perm + static_cast<long long>(head) * J.tokens;
  const T* xb = static_cast<const T*>(J.x) + static_cast<long long>(head) * J.head_rows * D + lane * E;
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.0f;
  if (J.big_rows > 0 && end - start > J.big_rows) return;  // a large cluster: the block kernel sums it
  bool bad = start < 0 || end > J.tokens || start > end;
  if (bad) end = start;
  auto token_id = [&](int pos) {
    int t = 0;
    if (pos < end) {
      t = perm[pos];
      if (t < 0 || t >= J.tokens) {
        bad = true;
        t = 0;
      }
    }
    return t;
  };
  int next_t = token_id(start + lane);
  for (int base = start; base < end; base += 32) {
    const int my_t = next_t;
    next_t = token_id(base + 32 + lane);
    const int cnt = min(32, end - base);
    for (int j = 0; j < cnt; j += kRows) {
      LaneRaw<T, E> v[kRows];
#pragma unroll
      for (int u = 0; u < kRows; ++u) {
        const int t = __shfl_sync(0xffffffffu, my_t, (j + u) & 31);
        if (j + u < cnt) v[u].load(xb + static_cast<long long>(t) * D);
      }
#pragma unroll
      for (int u = 0; u < kRows; ++u)
        if (j + u < cnt)
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = __fadd_rn(acc[e], v[u].get(e));
    }
  }
  if (bad && lane == 0) record_status(status, kDevBadIndex);
  const int n = end - start;
  const long long o = (static_cast<long long>(head) * J.clusters + c) * D + lane * E;
  float nsq = 0.0f;
  float mv[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float m = n > 0 ? __fdiv_rn(acc[e], static_cast<float>(n)) : J.previous[o + e];
    mv[e] = m;
    J.means[o + e] = m;
    if (J.sums) J.sums[o + e] = acc[e];
    nsq = fmaf(m, m, nsq);
  }
  if (J.image) {
    const CenterGeom g = center_geom(J.clusters, D);
    write_image<E>(J.image + static_cast<long long>(head) * g.nchunks * g.b_bytes, g, c, lane * E, mv);
  }
  if (J.norms) {
    nsq = warp_sum(nsq);
    if (lane == 0) J.norms[static_cast<long long>(head) * J.clusters + c] = nsq;
  }
}

// The same update with W warps per cluster (one block per cluster, bf16
// tokens), for calls with few heads: there every cluster's block is resident
// at once and the call waits for its largest cluster, whose rows the one-warp
// kernel fetches 16 per round trip.  Warp s owns elements [s D/W, (s+1) D/W),
// lane l the E = D/(32 W) of them from s D/W + l E; the narrower slice per
// lane lets every warp keep two 32-row batches in flight (the next batch
// loads while the current one is summed).  Each element is still summed over
// the cluster's tokens in ascending order, and the norm is reduced in the
// one-warp kernel's order (per lane of that kernel its D/32 elements, then the
// lanes by xor) from the means staged in shared memory, so every output is
// bit-identical to the one-warp kernel's.
template <int D, int W>
__global__ void __launch_bounds__(32 * W, 4) kmeans_update_wide_kernel(const UpdateJobs jobs, int bh,
                                                                       unsigned* status) {
  using T = __nv_bfloat16;
  constexpr int E = D / (32 * W);
  constexpr int kBatch = 32;
  static_assert(E >= 1 && E * 32 * W == D, "W must divide D / 32");
  const UpdateJob J = blockIdx.y ? jobs.job[1] : jobs.job[0];  // no dynamic index into the parameters
  const long long w = blockIdx.x;
  if (w >= static_cast<long long>(bh) * J.clusters) return;
  const int sub = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = static_cast<int>(w / J.clusters);
  const int c = static_cast<int>(w - static_cast<long long>(head) * J.clusters);
  const int start = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c];
  int end = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c + 1];
  if (J.big_rows > 0 && end - start > J.big_rows) return;  // the block kernel sums it
  bool bad = start < 0 || end > J.tokens || start > end;
  if (bad) end = start;
  const int32_t* perm = J.perm + static_cast<long long>(head) * J.tokens;
  const int d0 = sub * (D / W) + lane * E;
  const T* xb = static_cast<const T*>(J.x) + static_cast<long long>(head) * J.head_rows * D + d0;
  auto token_id = [&](int pos) {
    int t = 0;
    if (pos < end) {
      t = perm[pos];
      if (t < 0 || t >= J.tokens) {
        bad = true;
        t = 0;
      }
    }
    return t;
  };
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.0f;
  LaneRaw<T, E> va[kBatch], vb[kBatch];
  auto load = [&](LaneRaw<T, E>(&v)[kBatch], int ids, int base) {
    const int cnt = min(kBatch, end - base);
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int t = __shfl_sync(0xffffffffu, ids, u);
      if (u < cnt) v[u].load(xb + static_cast<long long>(t) * D);
    }
  };
  auto sum = [&](const LaneRaw<T, E>(&v)[kBatch], int base) {
    const int cnt = min(kBatch, end - base);
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (u < cnt)
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] = __fadd_rn(acc[e], v[u].get(e));
  };
  // batch b holds the tokens at positions [start + 32 b, start + 32 b + 32);
  // its ids are read two batches ahead, its rows one batch ahead
  int ids_next = token_id(start + kBatch + lane);
  load(va, token_id(start + lane), start);
  for (int base = start; base < end; base += 2 * kBatch) {
    int ids_after = token_id(base + 2 * kBatch + lane);
    if (base + kBatch < end) load(vb, ids_next, base + kBatch);
    sum(va, base);
    if (base + kBatch >= end) break;
    ids_next = token_id(base + 3 * kBatch + lane);
    if (base + 2 * kBatch < end) load(va, ids_after, base + 2 * kBatch);
    sum(vb, base + kBatch);
  }
  if (bad) record_status(status, kDevBadIndex);
  const int n = end - start;
  const long long o = (static_cast<long long>(head) * J.clusters + c) * D + d0;
  __shared__ float means[D];
  float mv[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float m = n > 0 ? __fdiv_rn(acc[e], static_cast<float>(n)) : J.previous[o + e];
    mv[e] = m;
    means[d0 + e] = m;
    J.means[o + e] = m;
    if (J.sums) J.sums[o + e] = acc[e];
  }
  if (J.image) {
    const CenterGeom g = center_geom(J.clusters, D);
    write_image<E>(J.image + static_cast<long long>(head) * g.nchunks * g.b_bytes, g, c, d0, mv);
  }
  if (J.norms) {
    __syncthreads();
    if (sub == 0) {
      constexpr int E1 = D / 32;
      float nsq = 0.0f;
#pragma unroll
      for (int e = 0; e < E1; ++e) nsq = fmaf(means[lane * E1 + e], means[lane * E1 + e], nsq);
      nsq = warp_sum(nsq);
      if (lane == 0) J.norms[static_cast<long long>(head) * J.clusters + c] = nsq;
    }
  }
}

// The clusters above J.big_rows rows (long sequences, bf16 tokens): one block
// of D threads per cluster, thread e owning element e.  The whole block loads
// kBigChunk rows per round trip into shared memory (the next chunk loads while
// the current one is summed), then every thread adds its element over those
// rows in token order -- the same sequence of fp32 additions, per element, as
// the warp kernel, so the result is identical.  The norm is reduced in the
// warp kernel's order (per lane its E elements, then the lanes by xor).
constexpr int kBigChunk = 64;
template <int D>
__global__ void __launch_bounds__(D) kmeans_update_big_kernel(const UpdateJobs jobs, int bh, unsigned* status) {
  using T = __nv_bfloat16;
  constexpr int E = D / 32;                        // the warp kernel's elements per lane
  constexpr int kRowVecs = D * 2 / 16;             // uint4 per row
  constexpr int kPer = kBigChunk * kRowVecs / D;   // uint4 per thread per chunk
  const UpdateJob J = blockIdx.y ? jobs.job[1] : jobs.job[0];  // no dynamic index into the parameters
  const long long w = blockIdx.x;
  if (J.big_rows <= 0 || w >= static_cast<long long>(bh) * J.clusters) return;
  const int head = static_cast<int>(w / J.clusters);
  const int c = static_cast<int>(w - static_cast<long long>(head) * J.clusters);
  const int start = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c];
  const int end = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c + 1];
  if (end - start <= J.big_rows) return;  // the warp kernel sums it
  if (start < 0 || end > J.tokens) {       // the warp kernel skipped it as large: report it here
    if (threadIdx.x == 0) record_status(status, kDevBadIndex);
    return;
  }
  __shared__ __align__(16) T buf[kBigChunk * D];
  __shared__ float part[32];
  const int e = threadIdx.x;
  const int32_t* perm = J.perm + static_cast<long long>(head) * J.tokens;
  const T* xb = static_cast<const T*>(J.x) + static_cast<long long>(head) * J.head_rows * D;
  bool bad = false;
  uint4 nxt[kPer];
  auto load_chunk = [&](int base) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int q = e + i * D, r = q / kRowVecs;
      nxt[i] = make_uint4(0, 0, 0, 0);
      if (base + r < end) {
        int t = perm[base + r];
        if (t < 0 || t >= J.tokens) {
          bad = true;
          t = 0;
        }
        nxt[i] = reinterpret_cast<const uint4*>(xb + static_cast<long long>(t) * D)[q % kRowVecs];
      }
    }
  };
  float acc = 0.0f;
  load_chunk(start);
  for (int base = start; base < end; base += kBigChunk) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) reinterpret_cast<uint4*>(buf)[e + i * D] = nxt[i];
    __syncthreads();
    if (base + kBigChunk < end) load_chunk(base + kBigChunk);  // in flight while this chunk is summed
    const int rows = min(kBigChunk, end - base);
    for (int r = 0; r < rows; ++r) acc = __fadd_rn(acc, to_f32<T>(buf[r * D + e]));
    __syncthreads();
  }
  if (bad) record_status(status, kDevBadIndex);
  const int n = end - start;
  const long long o = (static_cast<long long>(head) * J.clusters + c) * D + e;
  const float m = __fdiv_rn(acc, static_cast<float>(n));
  J.means[o] = m;
  if (J.sums) J.sums[o] = acc;
  if (J.image) {
    const CenterGeom g = center_geom(J.clusters, D);
    const float mv[1] = {m};
    write_image<1>(J.image + static_cast<long long>(head) * g.nchunks * g.b_bytes, g, c, e, mv);
  }
  if (J.norms) {
    // lane l of the warp kernel held elements [l E, (l + 1) E): its partial,
    // then the xor reduction over the 32 partials
    const unsigned grp = 0xffffffffu;
    float nsq = 0.0f;
#pragma unroll
    for (int k2 = 0; k2 < E; ++k2) {
      const float mk = __shfl_sync(grp, m, (threadIdx.x & 31 & ~(E - 1)) + k2);
      nsq = fmaf(mk, mk, nsq);
    }
    if ((e % E) == 0) part[e / E] = nsq;
    __syncthreads();
    if (threadIdx.x < 32) {
      const float v = warp_sum(part[threadIdx.x]);
      if (threadIdx.x == 0) J.norms[static_cast<long long>(head) * J.clusters + c] = v;
    }
  }
}

bool make_token_map(CUtensorMap* m, const void* base, long long rows, int dims) {
  const uint64_t gdims[2] = {static_cast<uint64_t>(dims), static_cast<uint64_t>(rows)};
  const uint64_t gstr[1] = {static_cast<uint64_t>(dims) * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(kTileM)};
  return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, gdims, gstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return kNumSMs;
  return n > 0 ? n : kNumSMs;
}

// x_hi/x_lo: bf16 token rows of each problem ([rows, D], head b at row
// b * head_rows; x_lo only in split mode), ``rows`` rows per map.
template <int D, bool SPLIT>
int launch_assign_t(AssignJobs jobs, const void* const (&x_hi)[2], const void* const (&x_lo)[2],
                    const long long (&rows)[2], cudaStream_t stream) {
  AssignMaps maps;
  for (int j = 0; j < jobs.njobs; ++j) {
    if (!make_token_map(&maps.xhi[j], x_hi[j], rows[j], D)) return kErrTensorMap;
    if (SPLIT && !make_token_map(&maps.xlo[j], x_lo[j], rows[j], D)) return kErrTensorMap;
  }
  if (jobs.njobs == 1) {
    maps.xhi[1] = maps.xhi[0];
    maps.xlo[1] = maps.xlo[0];
  }
  const AssignSmem S = assign_smem(jobs.job[0].clusters, jobs.njobs > 1 ? jobs.job[1].clusters : 1, jobs.njobs, D, SPLIT);
  if (S.smem > 227 * 1024) return kErrUnsupported;
  long long total_cost = 0;
  for (int j = 0; j < 2; ++j) {
    if (j < jobs.njobs) {
      const CenterGeom g = center_geom(jobs.job[j].clusters, D);
      jobs.items[j] = static_cast<long long>(jobs.bh) * ((jobs.job[j].tokens + kTileM - 1) / kTileM);
      // a token tile costs a fixed part (tile load, hand-offs, labels) plus a
      // part per centroid column; counting the fixed part (~410 columns'
      // worth, from per-tile periods at C = 128 and 256) moves CTAs from K to
      // Q groups.  Measured on HV-480: 12 heads -12 us per call (Q5/K7 CTAs
      // per head instead of Q4/K8), 6 heads +4-9 us, 3 and 24 heads no
      // change; so it is counted for 9-16 heads only
      jobs.cost[j] = (jobs.bh > 8 && jobs.bh <= 16 ? 410LL : 0LL) + static_cast<long long>(g.nchunks) * g.nc;
      total_cost += jobs.items[j] * jobs.cost[j];
    } else {
      jobs.items[j] = 0;
      jobs.cost[j] = 1;
    }
  }
  const long long items = jobs.items[0] + jobs.items[1];
  const int sms = sm_count();
  jobs.ncta = static_cast<int>(items < sms ? items : sms);
  jobs.split[0] = jobs.split[1] = 0;
  if (static_cast<long long>(jobs.bh) * jobs.njobs <= sms) {
    // CTAs per group in proportion to the group's cost, at most one CTA per SM
    long long ctas = 0;
    for (int j = 0; j < jobs.njobs; ++j) {
      const long long nt = (jobs.job[j].tokens + kTileM - 1) / kTileM;
      const long long share = nt * jobs.cost[j] * sms / total_cost;
      jobs.split[j] = static_cast<int>(share < 1 ? 1 : (share > nt ? nt : share));
      ctas += static_cast<long long>(jobs.bh) * jobs.split[j];
    }
    // with the fixed tile cost counted (9-16 heads), SMs left over go to the
    // group with the larger remainder, a CTA per head at a time
    for (int pass = 0; pass < 2 && jobs.bh > 8 && jobs.bh <= 16; ++pass) {
      int best = -1;
      long long best_frac = -1;
      for (int j = 0; j < jobs.njobs; ++j) {
        const long long nt = (jobs.job[j].tokens + kTileM - 1) / kTileM;
        const long long frac = (nt * jobs.cost[j] * sms) % total_cost;
        if (jobs.split[j] < nt && frac > best_frac) {
          best = j;
          best_frac = frac;
        }
      }
      if (best >= 0 && ctas + jobs.bh <= sms) {
        ++jobs.split[best];
        ctas += jobs.bh;
      }
    }
    if (ctas <= sms) jobs.ncta = static_cast<int>(ctas);
    else jobs.split[0] = jobs.split[1] = 0;
  }
  // one CTA per SM (its 512 TMEM columns are then always free); CTAs that
  // serve one resident group use the room left for a deeper token-tile ring
  int smem = S.smem > 116 * 1024 ? S.smem : 116 * 1024;
  if (jobs.split[0] > 0 && S.resident) {
    // the per-block opt-in limit less the kernel's static shared memory
    cudaFuncAttributes fa;
    int dev = 0, optin = 0;
    if (cudaFuncGetAttributes(&fa, kmeans_assign_kernel<D, SPLIT>) == cudaSuccess && cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess) {
      const int full = (optin - static_cast<int>(fa.sharedSizeBytes)) & ~1023;
      smem = full > smem ? full : smem;
    }
  }
  jobs.dyn_smem = smem;
  cudaError_t e = cudaFuncSetAttribute(kmeans_assign_kernel<D, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  kmeans_assign_kernel<D, SPLIT><<<jobs.ncta, kAssignThreads, smem, stream>>>(maps, jobs, device_status_ptr());
  return launch_status();
}

// norms and bf16 hi/lo image of [bh, C, D] centroids
// norms and image of one or two sets of centres, one launch
int launch_prep_jobs(const PrepJobs& jobs, int njobs, int bh, int dims, cudaStream_t stream) {
  long long blocks = 1;
  for (int j = 0; j < njobs; ++j) {
    const CenterGeom g = center_geom(jobs.job[j].C, dims);
    const long long b = (static_cast<long long>(bh) * g.nchunks * g.nc * 32 + 255) / 256;
    blocks = b > blocks ? b : blocks;
  }
  const dim3 grid(static_cast<unsigned>(blocks), njobs);
  if (dims == 128) center_prep_kernel<128><<<grid, 256, 0, stream>>>(jobs, bh);
  else if (dims == 64) center_prep_kernel<64><<<grid, 256, 0, stream>>>(jobs, bh);
  else return kErrUnsupported;
  return launch_status();
}

int launch_prep(const float* centers, float* norms, unsigned char* image, int bh, int C, int dims, cudaStream_t stream) {
  PrepJobs jobs{};
  jobs.job[0] = {centers, norms, image, C};
  return launch_prep_jobs(jobs, 1, bh, dims, stream);
}

long long image_bytes_per_head(int C, int dims) {
  const CenterGeom g = center_geom(C, dims);
  return static_cast<long long>(g.nchunks) * g.b_bytes;
}

// The wide update (two warps per cluster) pays off while every cluster's block
// is resident at once; measured on B200 at HV-480 shapes (Q 128 + K 256
// clusters per head): 3, 6 and 12 heads per call gain 60, 58 and 44 us per
// call, 24 heads (12288 clusters) none.
constexpr int kUpdateWideWarps = 2;
constexpr long long kUpdateWideMaxClusters = 8192;

template <typename T>
int launch_update_t(const UpdateJobs& jobs, int njobs, int bh, int dims, int max_clusters, cudaStream_t stream) {
  const long long warps = static_cast<long long>(bh) * max_clusters;
  // few clusters in all (few heads): a block of several warps per cluster
  constexpr int kWide = kUpdateWideWarps;
  bool wide = false;
  if constexpr (std::is_same<T, __nv_bfloat16>::value && kWide > 1) {
    wide = warps * njobs <= kUpdateWideMaxClusters;
    if (wide) {
      const dim3 wgrid(static_cast<unsigned>(warps), njobs);
      if (dims == 128)
        kmeans_update_wide_kernel<128, kWide><<<wgrid, 32 * kWide, 0, stream>>>(jobs, bh, device_status_ptr());
      else if (dims == 64)
        kmeans_update_wide_kernel<64, 2><<<wgrid, 64, 0, stream>>>(jobs, bh, device_status_ptr());
      else
        return kErrUnsupported;
    }
  }
  if (!wide) {
    dim3 grid(static_cast<unsigned>((warps * 32 + kUpdateThreads - 1) / kUpdateThreads), njobs);
    if (dims == 128) kmeans_update_kernel<128, T><<<grid, kUpdateThreads, 0, stream>>>(jobs, bh, device_status_ptr());
    else if (dims == 64) kmeans_update_kernel<64, T><<<grid, kUpdateThreads, 0, stream>>>(jobs, bh, device_status_ptr());
    else return kErrUnsupported;
  }
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    bool big = false;
    for (int j = 0; j < njobs; ++j) big = big || jobs.job[j].big_rows > 0;
    if (big) {
      const dim3 bgrid(static_cast<unsigned>(warps), njobs);  // a block per (head, cluster)
      if (dims == 128) kmeans_update_big_kernel<128><<<bgrid, 128, 0, stream>>>(jobs, bh, device_status_ptr());
      else kmeans_update_big_kernel<64><<<bgrid, 64, 0, stream>>>(jobs, bh, device_status_ptr());
    }
  }
  return launch_status();
}

}  // namespace

// ---------------------------------------------------------------------------
// fused fixed-iteration k-means over bf16 tokens (one or two independent
// problems per launch, e.g. the Q and K clusterings of one PECO call)
// ---------------------------------------------------------------------------
int kmeans_fit_bf16(int njobs, const KmeansProblem* probs, int bh, int dims, int iters, cudaStream_t stream) {
  if (njobs < 1 || njobs > 2 || bh < 1 || iters < 1) return kErrInvalidValue;
  if (dims != 64 && dims != 128) return kErrUnsupported;
  int rc = 0;
  int maxc = 0;
  const void* xs[2] = {probs[0].x, njobs > 1 ? probs[1].x : probs[0].x};
  const void* none[2] = {nullptr, nullptr};
  long long rows[2] = {0, 0};
  PrepJobs prep{};
  for (int j = 0; j < njobs; ++j) {
    const KmeansProblem& p = probs[j];
    if (p.clusters < 1 || p.tokens < 1 || p.clusters > p.tokens || p.head_rows < p.tokens) return kErrInvalidValue;
    if ((reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.image)) & 15) return kErrInvalidValue;
    maxc = max(maxc, p.clusters);
    // the token map covers every head's rows up to the last token
    rows[j] = static_cast<long long>(bh - 1) * p.head_rows + p.tokens;
    // norms and image of the initial centres (both problems in one launch below)
    prep.job[j] = {p.centers_a, p.norms, p.image, p.clusters};
  }
  rc = launch_prep_jobs(prep, njobs, bh, dims, stream);
  if (rc) return rc;
  for (int it = 0; it < iters; ++it) {
    AssignJobs aj{};
    aj.njobs = njobs;
    aj.bh = bh;
    UpdateJobs uj{};
    for (int j = 0; j < njobs; ++j) {
      const KmeansProblem& p = probs[j];
      // ping-pong so that the last iteration writes centers_out
      const bool even_left = ((iters - 1 - it) & 1) == 0;
      const float* cur = (it == 0) ? p.centers_a : (even_left ? p.centers_b : p.centers_out);
      float* nxt = even_left ? p.centers_out : p.centers_b;  // in-place is safe: each lane reads then writes
      // the first iteration records the token norms, later ones read them
      aj.job[j] = {p.tokens, p.clusters, p.head_rows, nullptr, static_cast<const __nv_bfloat16*>(p.x), cur, p.norms,
                   p.image, p.labels, it > 0 ? p.xnorm : nullptr, it == 0 ? p.xnorm : nullptr};
      // the last update needs no image: nothing assigns against it
      // long sequences: clusters above 512 rows go to the block kernel
      uj.job[j] = {p.x, p.head_rows, p.tokens, p.clusters, p.perm, p.offsets, cur, nxt, nullptr, p.norms,
                   it + 1 < iters ? p.image : nullptr, p.tokens >= 32768 ? 512 : 0};
    }
    rc = dims == 128 ? launch_assign_t<128, false>(aj, xs, none, rows, stream)
                     : launch_assign_t<64, false>(aj, xs, none, rows, stream);
    if (rc) return rc;
    SortJobInput sj[2];
    for (int j = 0; j < njobs; ++j) {
      const KmeansProblem& p = probs[j];
      sj[j] = {p.labels, p.tokens, bh, p.tokens, p.clusters, p.perm, p.counts, p.offsets, p.sort_seg,
               sort_segments(p.tokens)};
    }
    rc = launch_stable_sort_jobs(sj, njobs, stream);
    if (rc) return rc;
    rc = launch_update_t<__nv_bfloat16>(uj, njobs, bh, dims, maxc, stream);
    if (rc) return rc;
  }
  return 0;
}

long long kmeans_work_floats(int clusters, int dims, int tokens) {
  if (clusters < 1 || tokens < 1 || (dims != 64 && dims != 128)) return -1;
  return static_cast<long long>(clusters) * dims + image_bytes_per_head(clusters, dims) / 4 + tokens +
         static_cast<long long>(sort_segments(tokens)) * clusters;
}

}  // namespace peco

using namespace peco;

// Drop-in for peco/kernels/kmeans.cu:139-175.  ``scratch`` is not needed by the
// tensor-core path and is left untouched; ``center_norms`` receives ||c||^2.
// fp32 tokens are split into bf16 hi + lo rows and the centroids into their
// bf16 image in stream-ordered scratch of this call.
extern "C" int peco_assign_tokens_to_centers(const float* x, const float* centers, int32_t* labels, float* scratch,
                                             float* center_norms, int batch, int tokens, int dims, int clusters,
                                             int chunk_size, void* stream_ptr) {
  (void)scratch;
  (void)chunk_size;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (batch < 1 || tokens < 1 || clusters < 1 || dims < 1) return kErrInvalidValue;
  if (dims != 64 && dims != 128) return kErrUnsupported;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(centers)) & 15) return kErrInvalidValue;
  const long long rows = static_cast<long long>(batch) * tokens;
  const size_t half_bytes = static_cast<size_t>(rows) * dims * 2;
  const size_t img_bytes = static_cast<size_t>(batch) * image_bytes_per_head(clusters, dims);
  void* buf = nullptr;
  cudaError_t e = cudaMallocAsync(&buf, 2 * half_bytes + img_bytes, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  unsigned char* hi = static_cast<unsigned char*>(buf);
  unsigned char* lo = hi + half_bytes;
  unsigned char* img = lo + half_bytes;
  int rc = launch_prep(centers, center_norms, img, batch, clusters, dims, stream);
  if (!rc) {
    const long long n4 = rows * dims / 4;
    long long blocks = (n4 + 255) / 256;
    if (blocks > kNumSMs * 16) blocks = kNumSMs * 16;
    split_rows_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(reinterpret_cast<const float4*>(x),
                                                                    reinterpret_cast<uint2*>(hi),
                                                                    reinterpret_cast<uint2*>(lo), n4);
    rc = launch_status();
  }
  if (!rc) {
    AssignJobs jobs{};
    jobs.njobs = 1;
    jobs.bh = batch;
    jobs.job[0] = {tokens, clusters, tokens, x, nullptr, centers, center_norms, img, labels, nullptr, nullptr};
    const void* xh[2] = {hi, hi};
    const void* xl[2] = {lo, lo};
    const long long nrows[2] = {rows, rows};
    rc = dims == 128 ? launch_assign_t<128, true>(jobs, xh, xl, nrows, stream)
                     : launch_assign_t<64, true>(jobs, xh, xl, nrows, stream);
  }
  cudaError_t f = cudaFreeAsync(buf, stream);
  return rc ? rc : static_cast<int>(f);
}

// Drop-in for peco/kernels/kmeans.cu:179-196: writes sums, counts and means
// (empty clusters keep ``previous``).  The stable sort needs batch*tokens +
// batch*(clusters+1) ints of scratch, taken from the stream-ordered pool.
extern "C" int peco_recompute_cluster_centers(const float* x, const int32_t* labels, const float* previous,
                                              float* sums, int32_t* counts, float* means, int batch, int tokens,
                                              int dims, int clusters, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (batch < 1 || tokens < 1 || clusters < 1 || dims < 1) return kErrInvalidValue;
  if (dims != 64 && dims != 128) return kErrUnsupported;
  const size_t n_perm = static_cast<size_t>(batch) * tokens, n_off = static_cast<size_t>(batch) * (clusters + 1);
  void* scratch = nullptr;
  cudaError_t e = cudaMallocAsync(&scratch, (n_perm + n_off) * sizeof(int32_t), stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  int32_t* perm = static_cast<int32_t*>(scratch);
  int32_t* offsets = perm + n_perm;
  int rc = launch_stable_sort(labels, tokens, batch, tokens, clusters, perm, counts, offsets, stream);
  if (!rc) {
    UpdateJobs uj{};
    uj.job[0] = {x, tokens, tokens, clusters, perm, offsets, previous, means, sums, nullptr, nullptr};
    rc = launch_update_t<float>(uj, 1, batch, dims, clusters, stream);
  }
  cudaError_t f = cudaFreeAsync(scratch, stream);
  if (!rc && f != cudaSuccess) rc = static_cast<int>(f);
  return rc;
}

// The same sort + update as peco_recompute_cluster_centers, with its scratch
// in g_update_scratch instead of the stream-ordered pool, so the call makes no
// allocation of any kind.  The scratch address is looked up once per device
// (cudaGetSymbolAddress with that device current); the first call on a device
// does that lookup.  Calls that overlap on one device (other streams, other
// threads) share the scratch and race: the caller serialises them.
namespace {
constexpr long long kStaticUpdateInts = 1LL << 21;
constexpr int kStaticMaxDevices = 64;
int32_t* g_update_scratch_ptr[kStaticMaxDevices] = {};
std::mutex g_update_scratch_mutex;

int update_scratch(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kStaticMaxDevices) return kErrUnsupported;
  std::lock_guard<std::mutex> lock(g_update_scratch_mutex);
  if (!g_update_scratch_ptr[dev]) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_update_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    g_update_scratch_ptr[dev] = static_cast<int32_t*>(addr);
  }
  *out = g_update_scratch_ptr[dev];
  return 0;
}
}  // namespace

extern "C" int peco_recompute_cluster_centers_static(const float* x, const int32_t* labels, const float* previous,
                                                     float* sums, int32_t* counts, float* means, int batch,
                                                     int tokens, int dims, int clusters, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (batch < 1 || tokens < 1 || clusters < 1 || dims < 1) return kErrInvalidValue;
  if (dims != 64 && dims != 128) return kErrUnsupported;
  const long long n_perm = static_cast<long long>(batch) * tokens;
  const long long n_off = static_cast<long long>(batch) * (clusters + 1);
  if (n_perm + n_off > kStaticUpdateInts) return kErrCapacity;
  int32_t* scratch = nullptr;
  int rc = update_scratch(&scratch);
  if (rc) return rc;
  int32_t* perm = scratch;
  int32_t* offsets = scratch + n_perm;
  rc = launch_stable_sort(labels, tokens, batch, tokens, clusters, perm, counts, offsets, stream);
  if (!rc) {
    UpdateJobs uj{};
    uj.job[0] = {x, tokens, tokens, clusters, perm, offsets, previous, means, sums, nullptr, nullptr};
    rc = launch_update_t<float>(uj, 1, batch, dims, clusters, stream);
  }
  return rc;
}

extern "C" long long peco_recompute_cluster_centers_static_capacity(void) { return kStaticUpdateInts; }

extern "C" int peco_kmeans_fit(const void* q_x, long long q_head_rows, int q_tokens, int q_clusters, int32_t* q_labels,
                               const float* q_init, float* q_centers, float* q_work, float* q_norms, int32_t* q_counts,
                               int32_t* q_offsets, int32_t* q_perm, const void* k_x, long long k_head_rows, int k_tokens,
                               int k_clusters, int32_t* k_labels, const float* k_init, float* k_centers, float* k_work,
                               float* k_norms, int32_t* k_counts, int32_t* k_offsets, int32_t* k_perm, int bh, int dims,
                               int iters, void* stream) {
  // work per problem: [bh, C, D] ping-pong centres, the bh centroid images,
  // the [bh, tokens] token norms, then (long rows) the label sort's
  // [bh, segments, C] scratch
  auto image_of = [&](float* work, int clusters) {
    return work ? reinterpret_cast<unsigned char*>(work + static_cast<long long>(bh) * clusters * dims) : nullptr;
  };
  auto xnorm_of = [&](float* work, int clusters) {
    if (!work || clusters < 1 || (dims != 64 && dims != 128)) return static_cast<float*>(nullptr);
    return work + static_cast<long long>(bh) * clusters * dims + static_cast<long long>(bh) * (image_bytes_per_head(clusters, dims) / 4);
  };
  auto sort_seg_of = [&](float* work, int clusters, int tokens) {
    float* xn = xnorm_of(work, clusters);
    return xn && tokens > 0 && sort_segments(tokens) > 0 ? reinterpret_cast<int32_t*>(xn + static_cast<long long>(bh) * tokens)
                                                         : static_cast<int32_t*>(nullptr);
  };
  KmeansProblem p[2];
  p[0] = {q_x, q_head_rows, q_tokens, q_clusters, q_init, q_work, q_centers, q_norms, q_labels, q_counts, q_offsets, q_perm,
          image_of(q_work, q_clusters), xnorm_of(q_work, q_clusters), sort_seg_of(q_work, q_clusters, q_tokens)};
  p[1] = {k_x, k_head_rows, k_tokens, k_clusters, k_init, k_work, k_centers, k_norms, k_labels, k_counts, k_offsets, k_perm,
          image_of(k_work, k_clusters), xnorm_of(k_work, k_clusters), sort_seg_of(k_work, k_clusters, k_tokens)};
  const int njobs = k_x ? 2 : 1;
  return kmeans_fit_bf16(njobs, p, bh, dims, iters, static_cast<cudaStream_t>(stream));
}

extern "C" long long peco_kmeans_work_floats(int clusters, int dims, int tokens) {
  return peco::kmeans_work_floats(clusters, dims, tokens);
}
