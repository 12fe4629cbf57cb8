// Token reorder, stable counting sort and Base-Offset PE quantization.
//
// Memory-bound passes (HBM roofline): every row is moved with 16-byte vector
// accesses, one half-warp (D=128, bf16) per token row, and the fused
// quantize+gather pass reads each input row once and writes each packed row
// once.  Quantization arithmetic uses explicitly rounded IEEE intrinsics
// (__fsub_rn/__fdiv_rn/__fmul_rn/__fadd_rn, rintf) so no multiply-add is ever
// contracted; this reproduces the reference's fp32 torch evaluation bit for
// bit (peco/quantization.py:111-118, 134-136).
#include <cooperative_groups.h>

#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

// ---------------------------------------------------------------------------
// legacy reorder (peco/kernels/kmeans.cu:92-107, 200-217)
// ---------------------------------------------------------------------------
// Forward: out[bh, j] = in[bh, idx[bh, j]];  inverse: out[bh, idx[bh, j]] = in[bh, j].
// One thread moves one 16-byte chunk; rows are row_chunks chunks long.
template <bool INVERSE>
__global__ void reorder_rows_vec(const uint4* __restrict__ in, const int32_t* __restrict__ idx, uint4* __restrict__ out,
                                 int tokens, int row_chunks, long long total_chunks, unsigned* status) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total_chunks;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / row_chunks;
    const int c = static_cast<int>(i - row * row_chunks);
    const long long head = row / tokens;
    const int t = idx[row];
    if (t < 0 || t >= tokens) {
      if (c == 0) record_status(status, kDevBadIndex);
      continue;
    }
    const long long mapped = (head * tokens + t) * row_chunks + c;
    if (INVERSE) out[mapped] = in[i];
    else out[i] = in[mapped];
  }
}

template <typename T, bool INVERSE>
__global__ void reorder_rows_scalar(const T* __restrict__ in, const int32_t* __restrict__ idx, T* __restrict__ out,
                                    int tokens, int dims, long long total, unsigned* status) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / dims;
    const int d = static_cast<int>(i - row * dims);
    const long long head = row / tokens;
    const int t = idx[row];
    if (t < 0 || t >= tokens) {
      if (d == 0) record_status(status, kDevBadIndex);
      continue;
    }
    const long long mapped = (head * tokens + t) * dims + d;
    if (INVERSE) out[mapped] = in[i];
    else out[i] = in[mapped];
  }
}

inline int grid_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  const long long cap = static_cast<long long>(kNumSMs) * 16;
  return static_cast<int>(b < 1 ? 1 : (b > cap ? cap : b));
}

// ---------------------------------------------------------------------------
// stable counting sort of labels (the argsort of peco/clustering.py:105)
// ---------------------------------------------------------------------------
// A row's tokens are split into contiguous partitions, one warp each;
// per-partition label counts give every (partition, label) a base offset in
// label-major order, and each warp then places its tokens in ascending order.
// The result equals a stable argsort: within a label, lower token index first.
// Optionally also emits counts [C] and offsets [C+1].  A row is sorted by one
// thread-block cluster (sort_labels_cluster_kernel, one launch); a long row
// with segment scratch by the segmented kernels below (three launches).
constexpr int kSortThreads = 1024;

// Lanes of the warp holding the same label as this lane (labels in
// [0, 2^nbits), -1 = none), from one ballot per label bit plus one for the
// sign: a handful of single-cycle votes where __match_any_sync costs hundreds
// of cycles per call on sm_100a (measured: 14,000 cycles for 8 calls in each
// of 32 warps of one CTA, against 700 for the votes).
__device__ __forceinline__ unsigned match_label(int l, int nbits) {
  const unsigned none = __ballot_sync(0xffffffffu, l < 0);
  unsigned m = l < 0 ? none : ~none;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (l >> b) & 1;
    const unsigned bb = __ballot_sync(0xffffffffu, bit);
    m &= bit ? bb : ~bb;
  }
  return m;
}

struct SortJob {
  const int32_t* labels;
  long long label_stride;
  int rows, tokens, clusters, parts;
  int32_t* indices;
  int32_t* counts;
  int32_t* offsets;
  int segs;         // CTAs per row (1: the whole row in one CTA)
  int32_t* seg;     // segs > 1: [rows][segs][clusters] per-segment counts, then bases
};
struct SortJobs {
  SortJob job[2];   // blockIdx.y selects the job (the Q and K sorts of one k-means iteration)
};

// Long rows with segment scratch: the sort is split over J.segs CTAs per row,
// each owning a contiguous token range, in three launches: mode 1 writes each
// segment's label counts, the scan kernel turns them into per-(segment, label)
// bases (and the counts and offsets), mode 2 recounts per warp and places the
// segment's tokens.
__global__ void __launch_bounds__(kSortThreads) stable_sort_labels_kernel(const SortJobs jobs, int mode,
                                                                         unsigned* status) {
  const SortJob J = blockIdx.y ? jobs.job[1] : jobs.job[0];  // no dynamic index into the parameters
  const int segs = J.segs;
  const int row = static_cast<int>(blockIdx.x) / segs, seg = static_cast<int>(blockIdx.x) % segs;
  if (row >= J.rows) return;
  const int32_t* __restrict__ labels = J.labels;
  const long long label_stride = J.label_stride;
  const int tokens = J.tokens, clusters = J.clusters, parts = J.parts;
  int32_t* __restrict__ indices = J.indices;
  extern __shared__ int32_t sm[];
  int32_t* hist = sm;                         // [parts][clusters]
  int32_t* colsum = sm + parts * clusters;    // [clusters]
  const int32_t* lab = labels + row * label_stride;
  int32_t* out_idx = indices + static_cast<long long>(row) * tokens;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int nbits = clusters > 1 ? 32 - __clz(clusters - 1) : 0;

  for (int i = threadIdx.x; i < parts * clusters; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  // this CTA's tokens [r0, r1) (a multiple of 32 per segment), one partition per warp
  const int span = segs > 1 ? (((tokens + segs - 1) / segs + 31) & ~31) : tokens;
  const int r0 = min(tokens, seg * span), r1 = min(tokens, r0 + span);
  const int plen = (r1 - r0 + parts - 1) / parts;
  // The first kSortCache batches of each partition are loaded once, all in
  // flight together, and kept in registers for both passes (the labels of a
  // 6750-token head fit); longer partitions load the rest the same way, a
  // round trip per kSortCache batches.
  constexpr int kSortCache = 8;
  int cached[kSortCache];
  unsigned cached_peers[kSortCache];  // their match masks, computed once for both passes
  const int p0 = r0 + warp * plen, p1 = min(r1, p0 + plen);
  auto label_at = [&](int t, bool report) {
    int l = (t < p1) ? lab[t] : -1;
    if (l >= clusters || (t < p1 && l < 0)) {
      if (report) record_status(status, kDevBadIndex);
      l = -1;
    }
    return l;
  };
#pragma unroll
  for (int i = 0; i < kSortCache; ++i) cached[i] = (warp < parts) ? label_at(p0 + 32 * i + lane, true) : -1;
  // phase 1: per-partition histograms (warp-aggregated, no atomics: one leader per label)
  if (warp < parts) {
#pragma unroll
    for (int i = 0; i < kSortCache; ++i) {
      const int l = cached[i];
      const unsigned peers = match_label(l, nbits);
      cached_peers[i] = peers;
      if (l >= 0 && (peers & lt_mask) == 0) hist[warp * clusters + l] += __popc(peers);
      __syncwarp();
    }
    // longer partitions: the rest kSortCache batches per round trip
    for (int base = p0 + 32 * kSortCache; base < p1; base += 32 * kSortCache) {
      int lb[kSortCache];
#pragma unroll
      for (int i = 0; i < kSortCache; ++i) lb[i] = label_at(base + 32 * i + lane, true);
#pragma unroll
      for (int i = 0; i < kSortCache; ++i) {
        const int l = lb[i];
        const unsigned peers = match_label(l, nbits);
        if (l >= 0 && (peers & lt_mask) == 0) hist[warp * clusters + l] += __popc(peers);
        __syncwarp();
      }
    }
  }
  __syncthreads();
  // phase 2: column sums -> counts; exclusive scan over labels -> offsets
  for (int c = threadIdx.x; c < clusters; c += blockDim.x) {
    int s = 0;
    for (int p = 0; p < parts; ++p) s += hist[p * clusters + c];
    colsum[c] = s;
  }
  __syncthreads();
  int32_t* segrow = J.seg + (static_cast<long long>(row) * segs + seg) * clusters;
  if (mode == 1) {  // this segment's label counts
    for (int c = threadIdx.x; c < clusters; c += blockDim.x) segrow[c] = colsum[c];
    return;
  }
  // mode 2: bases from the scan; hist becomes per-partition base offsets
  for (int c = threadIdx.x; c < clusters; c += blockDim.x) {
    int b = segrow[c];
    for (int p = 0; p < parts; ++p) {
      const int h = hist[p * clusters + c];
      hist[p * clusters + c] = b;
      b += h;
    }
  }
  __syncthreads();
  // phase 3: stable placement
  if (warp < parts) {
    auto place = [&](int t, int l, unsigned peers) {
      int pos = 0;
      if (l >= 0) pos = hist[warp * clusters + l] + __popc(peers & lt_mask);
      __syncwarp();
      if (l >= 0) {
        out_idx[pos] = t;
        if ((peers & lt_mask) == 0) hist[warp * clusters + l] += __popc(peers);
      }
      __syncwarp();
    };
#pragma unroll
    for (int i = 0; i < kSortCache; ++i) place(p0 + 32 * i + lane, cached[i], cached_peers[i]);
    for (int base = p0 + 32 * kSortCache; base < p1; base += 32 * kSortCache) {
      int lb[kSortCache];
#pragma unroll
      for (int i = 0; i < kSortCache; ++i) lb[i] = label_at(base + 32 * i + lane, false);
#pragma unroll
      for (int i = 0; i < kSortCache; ++i) place(base + 32 * i + lane, lb[i], match_label(lb[i], nbits));
    }
  }
}

// Segmented sort, middle launch (one CTA per row): label totals over the
// segments -> counts and offsets, and each (segment, label) count replaced by
// its base position (label-major, then segment order, which keeps the sort
// stable).
__global__ void __launch_bounds__(kSortThreads) sort_segments_scan_kernel(const SortJobs jobs) {
  const SortJob J = blockIdx.y ? jobs.job[1] : jobs.job[0];
  const int row = blockIdx.x;
  if (row >= J.rows) return;
  const int clusters = J.clusters, segs = J.segs;
  extern __shared__ int32_t tot[];  // [clusters]
  __shared__ int32_t warp_tot[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* sg = J.seg + static_cast<long long>(row) * segs * clusters;
  for (int c = threadIdx.x; c < clusters; c += blockDim.x) {
    int t = 0;
    for (int g = 0; g < segs; ++g) t += sg[static_cast<long long>(g) * clusters + c];
    tot[c] = t;
  }
  __syncthreads();
  const int per = (clusters + blockDim.x - 1) / blockDim.x;
  const int c0 = threadIdx.x * per, c1 = min(clusters, c0 + per);
  int local = 0;
  for (int c = c0; c < c1; ++c) local += tot[c];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = warp_tot[lane];
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += u;
    }
    warp_tot[lane] = inc - v;  // exclusive warp offsets (the block has 32 warps)
  }
  __syncthreads();
  int run = warp_tot[warp] + incl - local;
  for (int c = c0; c < c1; ++c) {
    if (J.counts) J.counts[static_cast<long long>(row) * clusters + c] = tot[c];
    if (J.offsets) J.offsets[static_cast<long long>(row) * (clusters + 1) + c] = run;
    int b = run;
    for (int g = 0; g < segs; ++g) {
      const long long i = static_cast<long long>(g) * clusters + c;
      const int n = sg[i];
      sg[i] = b;
      b += n;
    }
    run += tot[c];
  }
  if (J.offsets && threadIdx.x == blockDim.x - 1) J.offsets[static_cast<long long>(row) * (clusters + 1) + clusters] = run;
}

// One row per thread-block cluster of kSortCluster CTAs, in one launch.  CTA s
// of the cluster owns the s-th contiguous segment of the row's tokens and
// each of its warps a contiguous partition of the segment.  The warps count
// their labels (shared memory), the CTA sums them into its segment's counts,
// and after a cluster barrier every CTA reads all segments' counts through
// distributed shared memory: label totals (their exclusive scan gives the
// offsets), and the counts of the segments before its own.  Base of
// (segment s, warp p, label c) = offset[c] + counts of c in segments < s +
// counts of c in warps < p of segment s: label-major, then token order, so
// the placement is the stable argsort.  A second cluster barrier keeps every
// CTA's counts alive until the other CTAs have read them.  Spreading a row
// over eight SMs is what makes the sort of a short row fast: the whole-row
// CTA above did all of a row's matching and scattered stores on one SM.
constexpr int kSortCluster = 8;
constexpr int kSortClusterThreads = 256;
constexpr int kSortClusterParts = kSortClusterThreads / 32;

__global__ void __cluster_dims__(kSortCluster, 1, 1) __launch_bounds__(kSortClusterThreads)
    sort_labels_cluster_kernel(const SortJobs jobs, unsigned* status) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const SortJob J = blockIdx.y ? jobs.job[1] : jobs.job[0];  // no dynamic index into the parameters
  const int row = static_cast<int>(blockIdx.x) / kSortCluster;
  if (row >= J.rows) return;  // the whole cluster (one row) leaves together
  const int seg = static_cast<int>(cl.block_rank());
  const int tokens = J.tokens, clusters = J.clusters;
  extern __shared__ int32_t sm[];
  int32_t* hist = sm;                                         // [parts][clusters]: counts, then bases
  int32_t* seg_count = sm + kSortClusterParts * clusters;     // [clusters]: this segment's counts
  int32_t* totals = seg_count + clusters;                     // [clusters]: the row's label counts
  int32_t* befores = totals + clusters;                       // [clusters]: counts in segments < seg
  __shared__ int32_t warp_tot[kSortClusterParts];
  const int32_t* lab = J.labels + row * J.label_stride;
  int32_t* out_idx = J.indices + static_cast<long long>(row) * tokens;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int nbits = clusters > 1 ? 32 - __clz(clusters - 1) : 0;
  for (int i = threadIdx.x; i < kSortClusterParts * clusters; i += blockDim.x) hist[i] = 0;
  const int span = (((tokens + kSortCluster - 1) / kSortCluster) + 31) & ~31;
  const int r0 = min(tokens, seg * span), r1 = min(tokens, r0 + span);
  const int plen = (r1 - r0 + kSortClusterParts - 1) / kSortClusterParts;
  const int p0 = r0 + warp * plen, p1 = min(r1, p0 + plen);
  auto label_at = [&](int t, bool report) {
    int l = (t < p1) ? lab[t] : -1;
    if (l >= clusters || (t < p1 && l < 0)) {
      if (report) record_status(status, kDevBadIndex);
      l = -1;
    }
    return l;
  };
  // the first kCache batches of the partition stay in registers (with their
  // match masks) for both passes; a longer partition re-reads the rest
  constexpr int kCache = 4;
  int cached[kCache];
  unsigned cached_peers[kCache];
#pragma unroll
  for (int i = 0; i < kCache; ++i) cached[i] = label_at(p0 + 32 * i + lane, true);
  __syncthreads();  // hist zeroed
  // phase 1: per-warp label counts (one leader lane per distinct label)
#pragma unroll
  for (int i = 0; i < kCache; ++i) {
    const int l = cached[i];
    const unsigned peers = match_label(l, nbits);
    cached_peers[i] = peers;
    if (l >= 0 && (peers & lt_mask) == 0) hist[warp * clusters + l] += __popc(peers);
    __syncwarp();
  }
  for (int base = p0 + 32 * kCache; base < p1; base += 32 * kCache) {
    int lb[kCache];
#pragma unroll
    for (int i = 0; i < kCache; ++i) lb[i] = label_at(base + 32 * i + lane, true);
#pragma unroll
    for (int i = 0; i < kCache; ++i) {
      const unsigned peers = match_label(lb[i], nbits);
      if (lb[i] >= 0 && (peers & lt_mask) == 0) hist[warp * clusters + lb[i]] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  // phase 2: this segment's label counts, published to the cluster
  for (int c = threadIdx.x; c < clusters; c += blockDim.x) {
    int s = 0;
#pragma unroll
    for (int p = 0; p < kSortClusterParts; ++p) s += hist[p * clusters + c];
    seg_count[c] = s;
  }
  cl.sync();
  // phase 3: label totals over the cluster's segments and the counts of the
  // segments before this one (each thread a contiguous run of labels); the
  // exclusive scan of the totals gives the offsets
  const int per = (clusters + blockDim.x - 1) / blockDim.x;
  const int c0 = min(clusters, static_cast<int>(threadIdx.x) * per), c1 = min(clusters, c0 + per);
  int local = 0;
  for (int c = c0; c < c1; ++c) {
    int tot = 0, before = 0;
#pragma unroll
    for (int g = 0; g < kSortCluster; ++g) {
      const int n = cl.map_shared_rank(seg_count, g)[c];
      tot += n;
      before += g < seg ? n : 0;
    }
    totals[c] = tot;
    befores[c] = before;
    local += tot;
  }
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int run = incl - local;  // exclusive prefix of c0 within the warp, plus the warps before
  for (int w2 = 0; w2 < warp; ++w2) run += warp_tot[w2];
  for (int c = c0; c < c1; ++c) {
    if (seg == 0) {
      if (J.counts) J.counts[static_cast<long long>(row) * clusters + c] = totals[c];
      if (J.offsets) J.offsets[static_cast<long long>(row) * (clusters + 1) + c] = run;
    }
    int b = run + befores[c];
#pragma unroll
    for (int p = 0; p < kSortClusterParts; ++p) {  // hist becomes per-warp bases
      const int h = hist[p * clusters + c];
      hist[p * clusters + c] = b;
      b += h;
    }
    run += totals[c];
  }
  if (seg == 0 && J.offsets && c1 == clusters && c0 < c1)
    J.offsets[static_cast<long long>(row) * (clusters + 1) + clusters] = run;
  // every CTA has read the others' counts; this CTA's bases are visible to its warps
  cl.sync();
  // phase 4: stable placement
  auto place = [&](int t, int l, unsigned peers) {
    int pos = 0;
    if (l >= 0) pos = hist[warp * clusters + l] + __popc(peers & lt_mask);
    __syncwarp();
    if (l >= 0) {
      out_idx[pos] = t;
      if ((peers & lt_mask) == 0) hist[warp * clusters + l] += __popc(peers);
    }
    __syncwarp();
  };
#pragma unroll
  for (int i = 0; i < kCache; ++i) place(p0 + 32 * i + lane, cached[i], cached_peers[i]);
  for (int base = p0 + 32 * kCache; base < p1; base += 32 * kCache) {
    int lb[kCache];
#pragma unroll
    for (int i = 0; i < kCache; ++i) lb[i] = label_at(base + 32 * i + lane, false);
#pragma unroll
    for (int i = 0; i < kCache; ++i) place(base + 32 * i + lane, lb[i], match_label(lb[i], nbits));
  }
}

// ---------------------------------------------------------------------------
// Base-Offset quantization of one token row (peco/quantization.py:96-136)
// ---------------------------------------------------------------------------
// A group of G lanes (G = D/8) holds one row, 8 consecutive elements per lane.
// Lanes of one row group: G consecutive lanes (G divides 32) handle one row.
// Groups of a warp may take different paths, so their shuffles name only
// their own lanes.
template <int G>
__device__ __forceinline__ unsigned row_group_mask() {
  if constexpr (G >= 32) {
    return 0xffffffffu;
  } else {
    return ((1u << G) - 1u) << ((threadIdx.x & 31) & ~(G - 1));
  }
}

template <int G>
struct RowQuant {
  // in: x[8], c[8] (fp32); out: xhat[8], code[8]; low/scale returned by ref.
  __device__ __forceinline__ static void run(const float (&x)[8], const float (&c)[8], float levels,
                                             float (&xhat)[8], float (&code)[8], float& low, float& scale) {
    // Every step is the reference's own fp32 operation rounded to nearest,
    // done two elements per instruction where sm_100 has a paired form
    // (x - c as x + (-c) is the same IEEE result).
    float2 r[4];
    float lo = INFINITY, hi = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      r[i] = fadd2(make_float2(x[2 * i], x[2 * i + 1]), make_float2(-c[2 * i], -c[2 * i + 1]));
      lo = fminf(lo, fminf(r[i].x, r[i].y));
      hi = fmaxf(hi, fmaxf(r[i].x, r[i].y));
    }
    const unsigned gmask = row_group_mask<G>();
#pragma unroll
    for (int o = G / 2; o; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(gmask, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(gmask, hi, o));
    }
    const float raw = __fdiv_rn(__fsub_rn(hi, lo), levels);
    const float sc = raw > 0.0f ? raw : 1.0f;
    // The code is rint(RN((r - lo) / sc)).  (r - lo) * (1/sc) is within a
    // few ulp of that quotient (< 2^-19 absolute for quotients <= 255), so
    // its rint is the same unless it sits within 1e-4 of a half-integer; only
    // then is the exact division evaluated.  r - lo >= 0 and 1/sc > 0, so
    // the code is never negative; the upper clamp is the reference's.
    const float inv = __frcp_rn(sc);
    const float2 nlo = make_float2(-lo, -lo), inv2 = make_float2(inv, inv);
    float2 num[4], q[4];
    bool exact = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      num[i] = fadd2(r[i], nlo);
      const float2 qa = fmul2(num[i], inv2);
      q[i] = make_float2(rintf(qa.x), rintf(qa.y));
      exact |= fabsf(qa.x - q[i].x) > 0.4999f || fabsf(qa.y - q[i].y) > 0.4999f;
    }
    if (exact) {  // rare: settle near-half quotients with the exact division
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        q[i].x = rintf(__fdiv_rn(num[i].x, sc));
        q[i].y = rintf(__fdiv_rn(num[i].y, sc));
      }
    }
    const float2 lo2 = make_float2(lo, lo);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = make_float2(fminf(q[i].x, levels), fminf(q[i].y, levels));
      code[2 * i] = q[i].x;
      code[2 * i + 1] = q[i].y;
      // x_hat = c + (low + scale * code), three separately rounded steps; the
      // product stays a scalar __fmul_rn, which is never fused into the add
      // that follows (a paired multiply feeding a paired add can be)
      const float2 prod = make_float2(__fmul_rn(sc, q[i].x), __fmul_rn(sc, q[i].y));
      const float2 xh = fadd2(make_float2(c[2 * i], c[2 * i + 1]), fadd2(lo2, prod));
      xhat[2 * i] = xh.x;
      xhat[2 * i + 1] = xh.y;
    }
    low = lo;
    scale = sc;
  }
};

template <typename T>
struct Vec8;  // 8 elements of T
template <>
struct Vec8<__nv_bfloat16> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec8<__half> {
  __device__ __forceinline__ static void load(const __half* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  __device__ __forceinline__ static void store(__half* p, const float (&v)[8]) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = pack_f16x2(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec8<float> {
  __device__ __forceinline__ static void load(const float* p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ __forceinline__ static void store(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

// Stand-alone Base-Offset pass over [BH, N, D]: mode 0 = fake quantize
// (write x_hat), mode 1 = encode (codes, low, scale), mode 2 = decode.
template <typename T, int D>
__global__ void base_offset_kernel(int mode, const T* __restrict__ x, const int32_t* __restrict__ labels,
                                   const float* __restrict__ centroids, T* __restrict__ out,
                                   uint8_t* __restrict__ codes, float* __restrict__ low_out,
                                   float* __restrict__ scale_out, int bh, int tokens, int clusters, int bits,
                                   unsigned* status) {
  constexpr int G = D / 8;
  const float levels = static_cast<float>((1 << bits) - 1);
  const long long rows = static_cast<long long>(bh) * tokens;
  const int sub = threadIdx.x % G;
  const long long first = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / G;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x / G;
  for (long long row = first; row < rows; row += step) {
    const long long head = row / tokens;
    int lab = labels[row];
    const bool bad = lab < 0 || lab >= clusters;
    if (bad) {
      if (sub == 0) record_status(status, kDevBadIndex);
      lab = 0;
    }
    const float* cen = centroids + (head * clusters + lab) * D + sub * 8;
    float c[8];
    {
      const float4 a = reinterpret_cast<const float4*>(cen)[0];
      const float4 b = reinterpret_cast<const float4*>(cen)[1];
      c[0] = a.x; c[1] = a.y; c[2] = a.z; c[3] = a.w;
      c[4] = b.x; c[5] = b.y; c[6] = b.z; c[7] = b.w;
    }
    float xh[8], q[8];
    if (mode == 2) {  // decode: x_hat = C[label] + (low + scale * code)
      const float lo = low_out[row], sc = scale_out[row];
      const uint2 cc = *reinterpret_cast<const uint2*>(codes + row * D + sub * 8);
      const uint8_t* cb = reinterpret_cast<const uint8_t*>(&cc);
#pragma unroll
      for (int i = 0; i < 8; ++i) xh[i] = __fadd_rn(c[i], __fadd_rn(lo, __fmul_rn(sc, static_cast<float>(cb[i]))));
      if (!bad) Vec8<T>::store(out + row * D + sub * 8, xh);
      continue;
    }
    float xv[8];
    Vec8<T>::load(x + row * D + sub * 8, xv);
    float lo, sc;
    RowQuant<G>::run(xv, c, levels, xh, q, lo, sc);
    if (bad) continue;
    if (mode == 0) {
      Vec8<T>::store(out + row * D + sub * 8, xh);
    } else {
      uint2 cc;
      uint8_t* cb = reinterpret_cast<uint8_t*>(&cc);
#pragma unroll
      for (int i = 0; i < 8; ++i) cb[i] = static_cast<uint8_t>(q[i]);
      *reinterpret_cast<uint2*>(codes + row * D + sub * 8) = cc;
      if (sub == 0) {
        low_out[row] = lo;
        scale_out[row] = sc;
      }
    }
  }
}

// Fused pass of one PECO call: for each of Q, K, V and each packed row j of
// a head, read source row perm[j] of the video tokens (x_hat for Q/K when
// bits > 0, plain copy for V), write it to packed row j; text rows (j >= Nv)
// are copied unchanged.  Q/K/V are [BH, S, D] with the video tokens first.
struct GatherJob {
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
  const int32_t* perm;       // [BH, Nv]
  const int32_t* labels;     // [BH, Nv] or null (no quantization)
  const float* centroids;    // [BH, C, D]
  int clusters;
};
struct GatherJobs {
  GatherJob job[3];
  // optional attention plan: K and V (jobs 1 and 2) then go to key blocks
  const int* plan;
  long long plan_stride, off_rows, blocks;
};

template <int D>
__global__ void __launch_bounds__(256, 6) quant_gather_kernel(GatherJobs jobs, int bh, int seq, int video, int bits,
                                                           unsigned* status) {
  constexpr int G = D / 8;  // lanes per row, 8 elements (16 bytes) each
  constexpr int R = 2;      // rows in flight per row group (with six blocks per SM: measured best)
  // no dynamic index into the kernel parameters (it would copy them to local memory)
  const GatherJob J = blockIdx.y == 0 ? jobs.job[0] : (blockIdx.y == 1 ? jobs.job[1] : jobs.job[2]);
  const bool to_blocks = jobs.plan && blockIdx.y > 0;
  const bool quant = J.labels && bits != 0;
  const float levels = static_cast<float>((1 << bits) - 1);
  const long long rows = static_cast<long long>(bh) * seq;
  const int sub = threadIdx.x % G;
  const long long first = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / G;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x / G;
  // rows advance by ``step``: keep (head, token) of the current row and add
  // step's own (head, token) split, so the loop never divides by seq
  const int step_h = static_cast<int>(step / seq);  // heads fit in int (bh <= 65535)
  const int step_j = static_cast<int>(step - static_cast<long long>(step_h) * seq);
  int h0 = static_cast<int>(first / seq);
  int j0 = static_cast<int>(first - static_cast<long long>(h0) * seq);
  auto advance = [&](int& h, int& jj) {
    h += step_h;
    jj += step_j;
    if (jj >= seq) {
      jj -= seq;
      ++h;
    }
  };
  for (long long r0 = first; r0 < rows; r0 += R * step) {
    // phase 1: destination row (key blocks for K/V) and source token of R rows
    int head[R], j[R], t[R], kr[R];
    bool live[R];
    int hu = h0;
    int ju = j0;
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const long long row = r0 + u * step;
      live[u] = row < rows;
      head[u] = live[u] ? hu : 0;
      j[u] = live[u] ? ju : 0;
      advance(hu, ju);  // row r0 + (u + 1) step
      if (u == R - 1) {
        h0 = hu;
        j0 = ju;
      }
      t[u] = j[u];
      kr[u] = j[u];
      if (live[u] && j[u] < video) t[u] = J.perm[static_cast<long long>(head[u]) * video + j[u]];
      if (live[u] && to_blocks) kr[u] = jobs.plan[static_cast<long long>(head[u]) * jobs.plan_stride + jobs.off_rows + j[u]];
    }
    // phase 2: source chunks and labels
    uint4 xr[R];
    int lab[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      lab[u] = 0;
      if (live[u] && (t[u] < 0 || t[u] >= (j[u] < video ? video : seq))) {
        if (sub == 0) record_status(status, kDevBadIndex);
        live[u] = false;
      }
      if (live[u] && to_blocks && kr[u] >= jobs.blocks * kKeyBlockRows) {
        if (sub == 0) record_status(status, kDevBadIndex);
        live[u] = false;
      }
      if (live[u] && to_blocks && kr[u] < 0) live[u] = false;  // key row outside every key cluster: never attended
      if (live[u]) {
        xr[u] = *reinterpret_cast<const uint4*>(J.src + (static_cast<long long>(head[u]) * seq + t[u]) * D + sub * 8);
        if (quant && j[u] < video) lab[u] = J.labels[static_cast<long long>(head[u]) * video + t[u]];
      }
    }
    // phase 3: centroid chunks, then quantise and store
#pragma unroll
    for (int u = 0; u < R; ++u) {
      if (!live[u]) continue;
      __nv_bfloat16* dst;
      if (to_blocks) {
        dst = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<unsigned char*>(J.dst) +
                                               (static_cast<long long>(head[u]) * jobs.blocks + kr[u] / kKeyBlockRows) * (kKeyBlockRows * D * 2) +
                                               key_block_offset(kr[u] % kKeyBlockRows, sub * 8));
      } else {
        dst = J.dst + (static_cast<long long>(head[u]) * seq + j[u]) * D + sub * 8;
      }
      if (!quant || j[u] >= video) {  // text rows and unquantised tensors: copy
        *reinterpret_cast<uint4*>(dst) = xr[u];
        continue;
      }
      if (lab[u] < 0 || lab[u] >= J.clusters) {
        if (sub == 0) record_status(status, kDevBadIndex);
        continue;
      }
      const float* cen = J.centroids + (static_cast<long long>(head[u]) * J.clusters + lab[u]) * D + sub * 8;
      float c[8], xv[8], xh[8], q[8];
      const float4 a = reinterpret_cast<const float4*>(cen)[0];
      const float4 b = reinterpret_cast<const float4*>(cen)[1];
      c[0] = a.x; c[1] = a.y; c[2] = a.z; c[3] = a.w;
      c[4] = b.x; c[5] = b.y; c[6] = b.z; c[7] = b.w;
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&xr[u]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        xv[2 * e] = f.x;
        xv[2 * e + 1] = f.y;
      }
      float lo, sc;
      RowQuant<G>::run(xv, c, levels, xh, q, lo, sc);
      Vec8<__nv_bfloat16>::store(dst, xh);
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
// Stable counting sorts of up to two label sets in one launch.
int launch_stable_sort_jobs(const SortJobInput* in, int njobs, cudaStream_t stream) {
  if (njobs < 1 || njobs > 2) return kErrInvalidValue;
  SortJobs jobs{};
  size_t smem = 0;
  int rows = 0, max_segs = 1, max_clusters = 1;
  bool segmented = true;
  for (int j = 0; j < njobs; ++j) {
    const SortJobInput& a = in[j];
    if (a.rows < 1 || a.tokens < 1 || a.clusters < 1) return kErrInvalidValue;
    int parts = 32;
    while (parts > 1 && static_cast<long long>(parts) * a.clusters * 4 + a.clusters * 4 > 160 * 1024) parts >>= 1;
    size_t need = (static_cast<size_t>(parts) * a.clusters + a.clusters) * sizeof(int32_t);
    if (need > 200 * 1024) return kErrUnsupported;
    const bool whole_row = !(a.seg && a.segs > 1);
    smem = need > smem ? need : smem;
    rows = a.rows > rows ? a.rows : rows;
    jobs.job[j] = {a.labels, a.label_stride, a.rows, a.tokens, a.clusters, parts, a.indices, a.counts, a.offsets,
                   whole_row ? 1 : a.segs, a.seg};
    segmented = segmented && a.seg && a.segs > 1;
    max_segs = a.segs > max_segs ? a.segs : max_segs;
    max_clusters = a.clusters > max_clusters ? a.clusters : max_clusters;
  }
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(stable_sort_labels_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  if (!segmented) {
    // one thread-block cluster per row
    const size_t csmem = static_cast<size_t>(kSortClusterParts + 3) * max_clusters * sizeof(int32_t);
    if (csmem > 200 * 1024) return kErrUnsupported;
    if (csmem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(sort_labels_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(csmem));
      if (e != cudaSuccess) return static_cast<int>(e);
    }
    sort_labels_cluster_kernel<<<dim3(static_cast<unsigned>(rows) * kSortCluster, njobs), kSortClusterThreads, csmem,
                                 stream>>>(jobs, device_status_ptr());
    return launch_status();
  }
  // long rows: segs CTAs per row (count, scan, place)
  const size_t scan_smem = static_cast<size_t>(max_clusters) * sizeof(int32_t);
  if (scan_smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(sort_segments_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(scan_smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  const dim3 grid(static_cast<unsigned>(rows) * max_segs, njobs);
  stable_sort_labels_kernel<<<grid, kSortThreads, smem, stream>>>(jobs, 1, device_status_ptr());
  sort_segments_scan_kernel<<<dim3(rows, njobs), kSortThreads, scan_smem, stream>>>(jobs);
  stable_sort_labels_kernel<<<grid, kSortThreads, smem, stream>>>(jobs, 2, device_status_ptr());
  return launch_status();
}

int launch_stable_sort(const int32_t* labels, long long label_stride, int rows, int tokens, int clusters,
                       int32_t* indices, int32_t* counts, int32_t* offsets, cudaStream_t stream) {
  const SortJobInput in = {labels, label_stride, rows, tokens, clusters, indices, counts, offsets};
  return launch_stable_sort_jobs(&in, 1, stream);
}

int launch_quant_gather(const void* q, const void* k, const void* v, void* qp, void* kp, void* vp,
                        const int32_t* q_perm, const int32_t* k_perm, const int32_t* q_labels,
                        const int32_t* k_labels, const float* q_cen, const float* k_cen, int cq, int ck, int bh,
                        int seq, int video, int dims, int bits, const int* plan, int gq, int gk,
                        cudaStream_t stream) {
  GatherJobs jobs;
  jobs.plan = plan;
  jobs.plan_stride = jobs.off_rows = jobs.blocks = 0;
  if (plan) {
    if (gq < 1 || gk < 1 || (reinterpret_cast<uintptr_t>(kp) | reinterpret_cast<uintptr_t>(vp)) & 15)
      return kErrInvalidValue;
    const PlanGeom g = plan_geom(seq, seq, gq, gk);
    jobs.plan_stride = g.stride;
    jobs.off_rows = g.off_rows;
    jobs.blocks = g.blocks;
  }
  jobs.job[0] = {static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(qp), q_perm,
                 bits ? q_labels : nullptr, q_cen, cq};
  jobs.job[1] = {static_cast<const __nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(kp), k_perm,
                 bits ? k_labels : nullptr, k_cen, ck};
  jobs.job[2] = {static_cast<const __nv_bfloat16*>(v), static_cast<__nv_bfloat16*>(vp), k_perm, nullptr, nullptr, 0};
  const long long rows = static_cast<long long>(bh) * seq;
  const int threads = 256;
  const int rows_per_block = threads / (dims / 8);
  long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  const long long cap = static_cast<long long>(kNumSMs) * 6;  // blocks per job: six resident per SM
  if (blocks > cap) blocks = cap;
  dim3 grid(static_cast<unsigned>(blocks), 3);
  if (dims == 128)
    quant_gather_kernel<128><<<grid, threads, 0, stream>>>(jobs, bh, seq, video, bits, device_status_ptr());
  else if (dims == 64)
    quant_gather_kernel<64><<<grid, threads, 0, stream>>>(jobs, bh, seq, video, bits, device_status_ptr());
  else
    return kErrUnsupported;
  return launch_status();
}

}  // namespace peco

using namespace peco;

extern "C" int peco_reorder_token_features(const void* input, const int32_t* indices, void* output,
                                           int batch_heads, int tokens, int dims, int item_size, int inverse,
                                           void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (batch_heads < 0 || tokens < 0 || dims < 0 || (item_size != 2 && item_size != 4)) return kErrInvalidValue;
  const long long total = static_cast<long long>(batch_heads) * tokens * dims;
  if (total == 0) return 0;
  const long long row_bytes = static_cast<long long>(dims) * item_size;
  const bool vec = (row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(input) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(output) % 16 == 0);
  unsigned* st = device_status_ptr();
  if (vec) {
    const int rc = static_cast<int>(row_bytes / 16);
    const long long chunks = static_cast<long long>(batch_heads) * tokens * rc;
    const int g = grid_for(chunks, 256);
    if (inverse)
      reorder_rows_vec<true><<<g, 256, 0, stream>>>(static_cast<const uint4*>(input), indices,
                                                    static_cast<uint4*>(output), tokens, rc, chunks, st);
    else
      reorder_rows_vec<false><<<g, 256, 0, stream>>>(static_cast<const uint4*>(input), indices,
                                                     static_cast<uint4*>(output), tokens, rc, chunks, st);
  } else {
    const int g = grid_for(total, 256);
    if (item_size == 2) {
      if (inverse)
        reorder_rows_scalar<uint16_t, true><<<g, 256, 0, stream>>>(static_cast<const uint16_t*>(input), indices,
                                                                  static_cast<uint16_t*>(output), tokens, dims,
                                                                  total, st);
      else
        reorder_rows_scalar<uint16_t, false><<<g, 256, 0, stream>>>(static_cast<const uint16_t*>(input), indices,
                                                                   static_cast<uint16_t*>(output), tokens, dims,
                                                                   total, st);
    } else {
      if (inverse)
        reorder_rows_scalar<uint32_t, true><<<g, 256, 0, stream>>>(static_cast<const uint32_t*>(input), indices,
                                                                  static_cast<uint32_t*>(output), tokens, dims,
                                                                  total, st);
      else
        reorder_rows_scalar<uint32_t, false><<<g, 256, 0, stream>>>(static_cast<const uint32_t*>(input), indices,
                                                                   static_cast<uint32_t*>(output), tokens, dims,
                                                                   total, st);
    }
  }
  return launch_status();
}

extern "C" int peco_sort_labels(const int32_t* labels, int32_t* indices, int32_t* counts, int32_t* offsets,
                                int rows, int tokens, int clusters, void* stream) {
  return launch_stable_sort(labels, tokens, rows, tokens, clusters, indices, counts, offsets,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int peco_base_offset(int mode, const void* x, const int32_t* labels, const float* centroids, void* out,
                                uint8_t* codes, float* offset_min, float* scale, int bh, int tokens, int dims,
                                int clusters, int bits, int dtype, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (mode < 0 || mode > 2 || bh < 0 || tokens < 0 || clusters < 1 || (bits != 4 && bits != 8))
    return kErrInvalidValue;
  if (dims != 64 && dims != 128) return kErrUnsupported;
  const long long rows = static_cast<long long>(bh) * tokens;
  if (rows == 0) return 0;
  const int threads = 256;
  const int rpb = threads / (dims / 8);
  long long blocks = (rows + rpb - 1) / rpb;
  const long long cap = static_cast<long long>(kNumSMs) * 8;
  if (blocks > cap) blocks = cap;
  unsigned* st = device_status_ptr();
#define PECO_BO_LAUNCH(T, DD)                                                                                \
  base_offset_kernel<T, DD><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(                          \
      mode, static_cast<const T*>(x), labels, centroids, static_cast<T*>(out), codes, offset_min, scale, bh, \
      tokens, clusters, bits, st)
  if (dtype == 0) {
    if (dims == 128) PECO_BO_LAUNCH(__half, 128); else PECO_BO_LAUNCH(__half, 64);
  } else if (dtype == 1) {
    if (dims == 128) PECO_BO_LAUNCH(__nv_bfloat16, 128); else PECO_BO_LAUNCH(__nv_bfloat16, 64);
  } else if (dtype == 2) {
    if (dims == 128) PECO_BO_LAUNCH(float, 128); else PECO_BO_LAUNCH(float, 64);
  } else {
    return kErrInvalidValue;
  }
#undef PECO_BO_LAUNCH
  return launch_status();
}

extern "C" int peco_quantize_gather(const void* q, const void* k, const void* v, void* q_packed, void* k_packed,
                                    void* v_packed, const int32_t* q_indices, const int32_t* k_indices,
                                    const int32_t* q_labels, const int32_t* k_labels, const float* q_centroids,
                                    const float* k_centroids, int q_clusters, int k_clusters, int bh, int seq,
                                    int video, int dims, int bits, const int* plan, int gq, int gk,
                                    void* stream) {
  if (bh < 1 || seq < 1 || video < 0 || video > seq || (bits != 0 && bits != 4 && bits != 8)) return kErrInvalidValue;
  return launch_quant_gather(q, k, v, q_packed, k_packed, v_packed, q_indices, k_indices, q_labels, k_labels,
                             q_centroids, k_centroids, q_clusters, k_clusters, bh, seq, video, dims, bits, plan, gq,
                             gk, static_cast<cudaStream_t>(stream));
}
