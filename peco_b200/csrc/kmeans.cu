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
// subtraction, with a 4x margin).  The epilogue keeps every centroid within
// 2E of the best one: a single survivor is the fp32 argmin outright; several
// survivors (near-ties) are recomputed exactly in fp32 on the CUDA cores and
// the lowest index wins ties.  Labels therefore equal the fp32 argmin except
// where two fp32 distances tie to rounding level.  fp32 inputs (the drop-in
// entry point) also split x into bf16 hi + lo (three MMA terms).
//
// Update (peco/kernels/kmeans.cu:179-196, peco/clustering.py:74-80): tokens
// are stably sorted by label (counting sort), then one warp per cluster sums
// its tokens in ascending token order in fp32 -- the accumulation order of the
// reference's CPU scatter_add -- and divides by the count; empty clusters keep
// their previous centre.  No atomics: the result is deterministic and, for
// identical labels, bit-identical to the reference's CPU centroids.
#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

#ifdef PECO_KMEANS_STATS
__device__ unsigned long long g_kstats[8];
#endif

constexpr int kTileM = 128;
constexpr int kProdWarps = 4, kEpiWarps = 4;
constexpr int kAssignThreads = 32 * (kProdWarps + 1 + kEpiWarps);
constexpr int kMaxCand = 8;
constexpr float kBoundScale = 2.44140625e-4f;   // 2^-12
constexpr float kBoundTiny = 9.5367431640625e-7f;  // 2^-20

struct AssignJob {
  const void* x;            // token rows, bf16 or fp32, row length D
  long long head_rows;      // rows between consecutive heads in x
  int tokens;               // tokens per head
  int clusters;             // centroids per head
  const float* centers;     // [B, C, D]
  const float* norms;       // [B, C] squared centroid norms
  int32_t* labels;          // [B, tokens]
};

struct AssignJobs {
  AssignJob job[2];
};

struct __align__(8) AssignBars {
  uint64_t a_full[2], a_empty[2], b_full[2], b_empty[2], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  float cmax;
};

__host__ __device__ constexpr int round16(int v) { return (v + 15) & ~15; }

struct AssignGeom {
  int nc;        // centroids per chunk (multiple of 16, <= 256)
  int nchunks;
  int a_bytes;   // one A slot: x as bf16 (hi [+ lo] for fp32 inputs)
  int b_bytes;   // one B slot: a centroid chunk as bf16 hi + lo
  int nbslots;   // B ring: 1 when the single chunk stays resident, else 2 (1 if smem is short)
  int naslots;   // A ring: 2 (1 if smem is short)
  int tmem_cols;
  int norms_off; // byte offset of the staged centroid norms
  int smem;      // dynamic smem bytes
};

__host__ __device__ inline AssignGeom assign_geom(int C, int D, bool xf32) {
  AssignGeom g;
  g.nc = round16(C < 256 ? C : 256);
  g.nchunks = (C + g.nc - 1) / g.nc;
  g.a_bytes = kTileM * D * 2 * (xf32 ? 2 : 1);
  g.b_bytes = 2 * g.nc * D * 2;
  g.nbslots = g.nchunks == 1 ? 1 : 2;
  g.naslots = 2;
  const int norm_bytes = ((C * 4) + 1023) & ~1023;
  while (1024 + g.nbslots * g.b_bytes + g.naslots * g.a_bytes + norm_bytes > 225 * 1024 &&
         (g.nbslots > 1 || g.naslots > 1)) {
    if (g.nbslots > 1) g.nbslots = 1;
    else g.naslots = 1;
  }
  int cols = 2 * g.nc;
  int p = 32;
  while (p < cols) p <<= 1;
  g.tmem_cols = p;
  g.norms_off = g.nbslots * g.b_bytes + g.naslots * g.a_bytes;
  g.smem = 1024 + g.norms_off + norm_bytes;
  return g;
}

// swizzled 16-byte chunk store into a K-major panel tile (panel = 64 columns,
// rows 128 bytes apart, ``panel_bytes`` between panels)
__device__ __forceinline__ void store_row_chunk(unsigned char* tile, int row, int chunk, uint4 v, int panel_bytes) {
  const int panel = chunk >> 3, c = chunk & 7;
  *reinterpret_cast<uint4*>(tile + panel * panel_bytes + row * 128 + ((c ^ (row & 7)) << 4)) = v;
}

__device__ __forceinline__ uint4 load_row_chunk(const unsigned char* tile, int row, int chunk, int panel_bytes) {
  const int panel = chunk >> 3, c = chunk & 7;
  return *reinterpret_cast<const uint4*>(tile + panel * panel_bytes + row * 128 + ((c ^ (row & 7)) << 4));
}

// bf16 hi/lo split of 8 fp32 values: hi = rn(v), lo = rn(v - hi)
__device__ __forceinline__ void split8(const float (&f)[8], uint4& hi, uint4& lo) {
  uint32_t* hw = reinterpret_cast<uint32_t*>(&hi);
  uint32_t* lw = reinterpret_cast<uint32_t*>(&lo);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float h0 = __bfloat162float(__float2bfloat16_rn(f[2 * e]));
    const float h1 = __bfloat162float(__float2bfloat16_rn(f[2 * e + 1]));
    hw[e] = pack_bf16x2(h0, h1);
    lw[e] = pack_bf16x2(f[2 * e] - h0, f[2 * e + 1] - h1);
  }
}

template <int D, bool XF32>
__global__ void __launch_bounds__(kAssignThreads, 1) kmeans_assign_kernel(const AssignJobs jobs, int tiles_per_cta,
                                                                        unsigned* status) {
  const AssignJob& J = jobs.job[blockIdx.z];
  const int head = blockIdx.y;
  const int C = J.clusters;
  const int ntiles = (J.tokens + kTileM - 1) / kTileM;
  const int t_begin = blockIdx.x * tiles_per_cta;
  if (t_begin >= ntiles) return;
  const int t_end = min(ntiles, t_begin + tiles_per_cta);
  const int my_tiles = t_end - t_begin;
  const AssignGeom G = assign_geom(C, D, XF32);

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* bslot[2] = {base, base + (G.nbslots > 1 ? G.b_bytes : 0)};
  unsigned char* aslot0 = base + G.nbslots * G.b_bytes;
  float* cn = reinterpret_cast<float*>(base + G.norms_off);  // squared centroid norms of this head
  __shared__ AssignBars sb;
  __shared__ float xnorm[2][kTileM];
  volatile int* abort_flag = &sb.abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* cen = J.centers + static_cast<long long>(head) * C * D;
  const float* norms = J.norms + static_cast<long long>(head) * C;
  const int NA = G.naslots, NB = G.nbslots;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sb.a_full[i], 32 * kProdWarps);
      mbar_init(&sb.a_empty[i], kEpiWarps);
      mbar_init(&sb.b_full[i], 32 * kProdWarps);
      mbar_init(&sb.b_empty[i], 1);
      mbar_init(&sb.acc_full[i], 1);
      mbar_init(&sb.acc_empty[i], kEpiWarps);
    }
    sb.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kProdWarps) {
    tmem_alloc(&sb.tmem_base, G.tmem_cols);
    tmem_relinquish();
  }
  for (int c = threadIdx.x; c < C; c += blockDim.x) cn[c] = norms[c];
  __syncthreads();
  // max centroid norm of this head (bound scale)
  if (warp == 0) {
    float m = 0.0f;
    for (int c = lane; c < C; c += 32) m = fmaxf(m, cn[c]);
    m = warp_max(m);
    if (lane == 0) sb.cmax = sqrtf(m);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;
  const int a_panel = kTileM * 128;         // bytes per 64-column panel of an A tile
  const int b_panel = G.nc * 128;           // bytes per 64-column panel of one B term
  const int b_term = G.nc * D * 2;          // offset of the lo term in a B slot

  if (warp < kProdWarps) {
    // ------------------------------------------------------------ producers
    const int tid = threadIdx.x;  // 0..127
    bool ok = true;
    auto load_b = [&](int chunk, unsigned char* dst) {
      // centroid rows j = tid, tid + 128 of this chunk, fp32 -> bf16 hi + lo
      for (int j = tid; j < G.nc; j += 32 * kProdWarps) {
        const int c = chunk * G.nc + j;
        const float4* src = reinterpret_cast<const float4*>(cen + static_cast<long long>(c) * D);
#pragma unroll
        for (int g = 0; g < D / 64; ++g) {
          float4 buf[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) buf[u] = c < C ? src[g * 16 + u] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float f[8] = {buf[2 * u].x, buf[2 * u].y, buf[2 * u].z, buf[2 * u].w,
                                buf[2 * u + 1].x, buf[2 * u + 1].y, buf[2 * u + 1].z, buf[2 * u + 1].w};
            uint4 hi, lo;
            split8(f, hi, lo);
            store_row_chunk(dst, j, g * 8 + u, hi, b_panel);
            store_row_chunk(dst + b_term, j, g * 8 + u, lo, b_panel);
          }
        }
      }
      fence_async_smem();
    };
    if (G.nchunks == 1) {
      load_b(0, bslot[0]);
      mbar_arrive(&sb.b_full[0]);
    }
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int tile = t_begin + i;
      const int s = i % NA, use = i / NA;
      if (use > 0) ok = mbar_wait_warp(&sb.a_empty[s], (use - 1) & 1, abort_flag, status);
      if (!ok) break;
      unsigned char* a_hi = aslot0 + s * G.a_bytes;
      unsigned char* a_lo = a_hi + kTileM * D * 2;
      const int row = tid;
      const int tok = tile * kTileM + row;
      float ss = 0.0f;
      if (tok < J.tokens) {
        const long long grow = static_cast<long long>(head) * J.head_rows + tok;
        if (XF32) {
          const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(J.x) + grow * D);
#pragma unroll
          for (int g = 0; g < D / 64; ++g) {
            float4 buf[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) buf[u] = src[g * 16 + u];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const float f[8] = {buf[2 * u].x, buf[2 * u].y, buf[2 * u].z, buf[2 * u].w,
                                  buf[2 * u + 1].x, buf[2 * u + 1].y, buf[2 * u + 1].z, buf[2 * u + 1].w};
#pragma unroll
              for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
              uint4 hi, lo;
              split8(f, hi, lo);
              store_row_chunk(a_hi, row, g * 8 + u, hi, a_panel);
              store_row_chunk(a_lo, row, g * 8 + u, lo, a_panel);
            }
          }
        } else {
          const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(J.x) + grow * D);
          uint4 buf[D / 8];
#pragma unroll
          for (int ch = 0; ch < D / 8; ++ch) buf[ch] = src[ch];
#pragma unroll
          for (int ch = 0; ch < D / 8; ++ch) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&buf[ch]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]);
              ss = fmaf(f.x, f.x, ss);
              ss = fmaf(f.y, f.y, ss);
            }
            store_row_chunk(a_hi, row, ch, buf[ch], a_panel);
          }
        }
      } else {
        for (int ch = 0; ch < D / 8; ++ch) {
          store_row_chunk(a_hi, row, ch, make_uint4(0, 0, 0, 0), a_panel);
          if (XF32) store_row_chunk(a_lo, row, ch, make_uint4(0, 0, 0, 0), a_panel);
        }
      }
      xnorm[s][row] = sqrtf(ss);
      fence_async_smem();
      mbar_arrive(&sb.a_full[s]);
      if (G.nchunks > 1) {
        for (int k = 0; k < G.nchunks && ok; ++k) {
          const int g = i * G.nchunks + k;
          const int bs = g % NB, bu = g / NB;
          if (bu > 0) ok = mbar_wait_warp(&sb.b_empty[bs], (bu - 1) & 1, abort_flag, status);
          if (!ok) break;
          load_b(k, bslot[bs]);
          mbar_arrive(&sb.b_full[bs]);
        }
      }
    }
  } else if (warp == kProdWarps) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc = instr_desc(128, G.nc, 1, false, false);
      bool ok = true;
      int last_g = -1;
      if (G.nchunks == 1) ok = mbar_wait(&sb.b_full[0], 0, abort_flag, status);
      for (int i = 0; i < my_tiles && ok; ++i) {
        const int s = i % NA;
        ok = mbar_wait(&sb.a_full[s], (i / NA) & 1, abort_flag, status);
        if (!ok) break;
        const uint32_t a_hi = smem_u32(aslot0 + s * G.a_bytes);
        const uint32_t a_lo = a_hi + kTileM * D * 2;
        for (int k = 0; k < G.nchunks && ok; ++k) {
          const int g = i * G.nchunks + k;
          const int as = g & 1, au = g >> 1;
          if (au > 0) ok = mbar_wait(&sb.acc_empty[as], (au - 1) & 1, abort_flag, status);
          int bs = 0;
          if (ok && G.nchunks > 1) {
            bs = g % NB;
            ok = mbar_wait(&sb.b_full[bs], (g / NB) & 1, abort_flag, status);
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t b_hi = smem_u32(bslot[bs]);
          const uint32_t b_lo = b_hi + b_term;
          const uint32_t acc = tmem + as * G.nc;
          // terms, smallest first: x.c_lo, [x_lo.c_hi], x.c_hi
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off_a = (kk >> 2) * a_panel + (kk & 3) * 32;
            const uint32_t off_b = (kk >> 2) * b_panel + (kk & 3) * 32;
            umma_ss(acc, smem_desc(a_hi + off_a, 16, 1024), smem_desc(b_lo + off_b, 16, 1024), idesc, kk > 0 ? 1u : 0u);
          }
          if (XF32) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off_a = (kk >> 2) * a_panel + (kk & 3) * 32;
              const uint32_t off_b = (kk >> 2) * b_panel + (kk & 3) * 32;
              umma_ss(acc, smem_desc(a_lo + off_a, 16, 1024), smem_desc(b_hi + off_b, 16, 1024), idesc, 1u);
            }
          }
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off_a = (kk >> 2) * a_panel + (kk & 3) * 32;
            const uint32_t off_b = (kk >> 2) * b_panel + (kk & 3) * 32;
            umma_ss(acc, smem_desc(a_hi + off_a, 16, 1024), smem_desc(b_hi + off_b, 16, 1024), idesc, 1u);
          }
          umma_commit(&sb.acc_full[as]);
          if (G.nchunks > 1) umma_commit(&sb.b_empty[bs]);
          last_g = g;
        }
      }
      if (last_g >= 0) mbar_wait(&sb.acc_full[last_g & 1], (last_g >> 1) & 1, abort_flag, status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float cmax = sb.cmax;
    bool ok = true;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int tile = t_begin + i;
      const int s = i % NA;
      ok = mbar_wait_warp(&sb.a_full[s], (i / NA) & 1, abort_flag, status);
      if (!ok) break;
      const float xn = xnorm[s][r];
      const float E2 = 2.0f * (kBoundScale * xn * cmax + kBoundTiny * (cmax * cmax + 2.0f * xn * cmax));
      float best = INFINITY;
      float cd[kMaxCand];
      int ci[kMaxCand];
      int ncand = 0;
      bool overflow = false;
      // keep entries within ``t`` (order preserved: slot m <= q)
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
      for (int k = 0; k < G.nchunks && ok; ++k) {
        const int g = i * G.nchunks + k;
        const int as = g & 1;
        ok = mbar_wait_warp(&sb.acc_full[as], (g >> 1) & 1, abort_flag, status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + as * G.nc + lane_off;
        for (int c0 = 0; c0 < G.nc; c0 += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32_sync(acc + c0, v);
          const int cb = k * G.nc + c0;
          float d[32];
          float mn = INFINITY;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int c = cb + j;
            d[j] = (c < C) ? fmaf(-2.0f, __uint_as_float(v[j]), cn[c]) : INFINITY;
            mn = fminf(mn, d[j]);
          }
          best = fminf(best, mn);
          const float thr = best + E2;
          // Candidates of this block as a bit mask; the (rare) pushes run in
          // one compact loop instead of 32 unrolled copies.
          unsigned m = 0;
          if (mn <= thr) {
#pragma unroll
            for (int j = 0; j < 32; ++j) m |= (d[j] <= thr ? 1u : 0u) << j;
          }
          while (m) {
            const int j = __ffs(m) - 1;
            m &= m - 1;
            float dj = 0.0f;
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) dj = (jj == j) ? d[jj] : dj;
            if (ncand == kMaxCand) prune(thr);
            if (ncand < kMaxCand) {
#pragma unroll
              for (int q = 0; q < kMaxCand; ++q)
                if (q == ncand) {
                  cd[q] = dj;
                  ci[q] = cb + j;
                }
              ++ncand;
            } else {
              overflow = true;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sb.acc_empty[as]);
      }
      if (!ok) break;
      const int tok = tile * kTileM + r;
      const bool valid = tok < J.tokens;
      prune(best + E2);
      int label = ncand > 0 ? ci[0] : 0;
      // Near-ties are recomputed in exact fp32, one token at a time by the
      // whole warp: lane l owns D/32 consecutive dimensions, so each
      // candidate centroid row is one coalesced load, and all candidates of
      // the token are in flight together.
      unsigned amb = __ballot_sync(0xffffffffu, valid && (overflow || ncand > 1));
      constexpr int E = D / 32;
      const unsigned char* a_hi = aslot0 + s * G.a_bytes;
      while (amb) {
        const int src = __ffs(amb) - 1;
        amb &= amb - 1;
        const int stok = __shfl_sync(0xffffffffu, tok, src);
        const int n = __shfl_sync(0xffffffffu, overflow ? -1 : ncand, src);
        const long long grow = static_cast<long long>(head) * J.head_rows + stok;
        float xv[E];
        if (XF32) {
          const float* xr = static_cast<const float*>(J.x) + grow * D + lane * E;
#pragma unroll
          for (int e = 0; e < E; ++e) xv[e] = xr[e];
        } else {
          const int srow = quarter * 32 + src;
          const uint4 u = load_row_chunk(a_hi, srow, (lane * E) >> 3, a_panel);
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u) + ((lane * E) & 7);
#pragma unroll
          for (int e = 0; e < E; ++e) xv[e] = __bfloat162float(h[e]);
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
      if (valid) {
        J.labels[static_cast<long long>(head) * J.tokens + tok] = label;
#ifdef PECO_KMEANS_STATS
        // debug builds: [0] tokens, [1] survivors after pruning, [2] overflows, [3] tokens needing a recompute
        atomicAdd(&g_kstats[0], 1ull);
        atomicAdd(&g_kstats[1], static_cast<unsigned long long>(ncand));
        if (overflow) atomicAdd(&g_kstats[2], 1ull);
        if (ncand > 1) atomicAdd(&g_kstats[3], 1ull);
#endif
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sb.a_empty[s]);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kProdWarps) {
    tc_fence_after();
    tmem_dealloc(tmem, G.tmem_cols);
  }
}

// ||c||^2 per centroid (fp32, one warp per centroid); writes norms [rows].
__global__ void center_norms_kernel(const float* __restrict__ centers, float* __restrict__ norms, long long rows,
                                    int dims) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const float* c = centers + w * dims;
  float s = 0.0f;
  for (int d = lane; d < dims; d += 32) s = fmaf(c[d], c[d], s);
  s = warp_sum(s);
  if (lane == 0) norms[w] = s;
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

template <int D, typename T>
__global__ void kmeans_update_kernel(const UpdateJobs jobs, int bh, unsigned* status) {
  const UpdateJob& J = jobs.job[blockIdx.y];
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(bh) * J.clusters) return;
  const int head = static_cast<int>(w / J.clusters);
  const int c = static_cast<int>(w - static_cast<long long>(head) * J.clusters);
  constexpr int E = D / 32;  // elements per lane
  const int start = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c];
  int end = J.offsets[static_cast<long long>(head) * (J.clusters + 1) + c + 1];
  const int32_t* perm = J.perm + static_cast<long long>(head) * J.tokens;
  const T* xb = static_cast<const T*>(J.x) + static_cast<long long>(head) * J.head_rows * D + lane * E;
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.0f;
  bool bad = start < 0 || end > J.tokens || start > end;
  if (bad) end = start;
  // The cluster's token ids arrive 32 at a time in one coalesced load; rows
  // are then fetched 8 at a time (all in flight) and added strictly in
  // ascending token order.
  for (int base = start; base < end; base += 32) {
    int my_t = 0;
    if (base + lane < end) {
      my_t = perm[base + lane];
      if (my_t < 0 || my_t >= J.tokens) {
        bad = true;
        my_t = 0;
      }
    }
    const int cnt = min(32, end - base);
    for (int j = 0; j < cnt; j += 8) {
      float v[8][E];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int t = __shfl_sync(0xffffffffu, my_t, (j + u) & 31);
        if (j + u < cnt) {
          const T* row = xb + static_cast<long long>(t) * D;
          load_lane_elems<T, E>(row, v[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (j + u < cnt)
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = __fadd_rn(acc[e], v[u][e]);
    }
  }
  if (bad && lane == 0) record_status(status, kDevBadIndex);
  const int n = end - start;
  const long long o = (static_cast<long long>(head) * J.clusters + c) * D + lane * E;
  float nsq = 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float m = n > 0 ? __fdiv_rn(acc[e], static_cast<float>(n)) : J.previous[o + e];
    J.means[o + e] = m;
    if (J.sums) J.sums[o + e] = acc[e];
    nsq = fmaf(m, m, nsq);
  }
  if (J.norms) {
    nsq = warp_sum(nsq);
    if (lane == 0) J.norms[static_cast<long long>(head) * J.clusters + c] = nsq;
  }
}

template <int D, bool XF32>
int launch_assign_t(const AssignJobs& jobs, int njobs, int bh, cudaStream_t stream) {
  int max_smem = 0, max_chunks = 0, max_tiles = 0;
  for (int j = 0; j < njobs; ++j) {
    const AssignGeom g = assign_geom(jobs.job[j].clusters, D, XF32);
    max_smem = max(max_smem, g.smem);
    max_chunks = max(max_chunks, g.nchunks);
    max_tiles = max(max_tiles, (jobs.job[j].tokens + kTileM - 1) / kTileM);
  }
  if (max_smem > 227 * 1024) return kErrUnsupported;
  // spread tiles so that ~2 waves of CTAs cover every (job, head)
  long long ctas_wanted = 2LL * kNumSMs;
  int per_head = static_cast<int>((ctas_wanted + static_cast<long long>(bh) * njobs - 1) / (static_cast<long long>(bh) * njobs));
  per_head = max(1, min(per_head, max_tiles));
  int tiles_per_cta = (max_tiles + per_head - 1) / per_head;
  if (max_chunks == 1) tiles_per_cta = max(tiles_per_cta, 2);  // amortise the resident centroid load
  const int grid_x = (max_tiles + tiles_per_cta - 1) / tiles_per_cta;
  cudaError_t e = cudaFuncSetAttribute(kmeans_assign_kernel<D, XF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid(grid_x, bh, njobs);
  kmeans_assign_kernel<D, XF32><<<grid, kAssignThreads, max_smem, stream>>>(jobs, tiles_per_cta, device_status_ptr());
  return launch_status();
}

int launch_norms(const float* centers, float* norms, long long rows, int dims, cudaStream_t stream) {
  const long long threads = rows * 32;
  const int blocks = static_cast<int>((threads + 255) / 256);
  center_norms_kernel<<<blocks, 256, 0, stream>>>(centers, norms, rows, dims);
  return launch_status();
}

template <typename T>
int launch_update_t(const UpdateJobs& jobs, int njobs, int bh, int dims, int max_clusters, cudaStream_t stream) {
  const long long warps = static_cast<long long>(bh) * max_clusters;
  dim3 grid(static_cast<unsigned>((warps * 32 + 255) / 256), njobs);
  if (dims == 128) kmeans_update_kernel<128, T><<<grid, 256, 0, stream>>>(jobs, bh, device_status_ptr());
  else if (dims == 64) kmeans_update_kernel<64, T><<<grid, 256, 0, stream>>>(jobs, bh, device_status_ptr());
  else return kErrUnsupported;
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
  for (int j = 0; j < njobs; ++j) {
    const KmeansProblem& p = probs[j];
    if (p.clusters < 1 || p.tokens < 1 || p.clusters > p.tokens) return kErrInvalidValue;
    maxc = max(maxc, p.clusters);
    // norms of the initial centres
    rc = launch_norms(p.centers_a, p.norms, static_cast<long long>(bh) * p.clusters, dims, stream);
    if (rc) return rc;
  }
  for (int it = 0; it < iters; ++it) {
    AssignJobs aj{};
    UpdateJobs uj{};
    for (int j = 0; j < njobs; ++j) {
      const KmeansProblem& p = probs[j];
      // ping-pong so that the last iteration writes centers_out
      const bool even_left = ((iters - 1 - it) & 1) == 0;
      const float* cur = (it == 0) ? p.centers_a : (even_left ? p.centers_b : p.centers_out);
      float* nxt = even_left ? p.centers_out : p.centers_b;  // in-place is safe: each lane reads then writes
      aj.job[j] = {p.x, p.head_rows, p.tokens, p.clusters, cur, p.norms, p.labels};
      uj.job[j] = {p.x, p.head_rows, p.tokens, p.clusters, p.perm, p.offsets, cur, nxt, nullptr, p.norms};
    }
    rc = dims == 128 ? launch_assign_t<128, false>(aj, njobs, bh, stream) : launch_assign_t<64, false>(aj, njobs, bh, stream);
    if (rc) return rc;
    for (int j = 0; j < njobs; ++j) {
      const KmeansProblem& p = probs[j];
      rc = launch_stable_sort(p.labels, p.tokens, bh, p.tokens, p.clusters, p.perm, p.counts, p.offsets, stream);
      if (rc) return rc;
    }
    rc = launch_update_t<__nv_bfloat16>(uj, njobs, bh, dims, maxc, stream);
    if (rc) return rc;
  }
  return 0;
}

}  // namespace peco

using namespace peco;

// Drop-in for peco/kernels/kmeans.cu:139-175.  ``scratch`` is not needed by the
// tensor-core path and is left untouched; ``center_norms`` receives ||c||^2.
extern "C" int peco_assign_tokens_to_centers(const float* x, const float* centers, int32_t* labels, float* scratch,
                                             float* center_norms, int batch, int tokens, int dims, int clusters,
                                             int chunk_size, void* stream_ptr) {
  (void)scratch;
  (void)chunk_size;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (batch < 1 || tokens < 1 || clusters < 1 || dims < 1) return kErrInvalidValue;
  if (dims != 64 && dims != 128) return kErrUnsupported;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(centers)) & 15) return kErrInvalidValue;
  int rc = launch_norms(centers, center_norms, static_cast<long long>(batch) * clusters, dims, stream);
  if (rc) return rc;
  AssignJobs jobs{};
  jobs.job[0] = {x, tokens, tokens, clusters, centers, center_norms, labels};
  return dims == 128 ? launch_assign_t<128, true>(jobs, 1, batch, stream) : launch_assign_t<64, true>(jobs, 1, batch, stream);
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
    uj.job[0] = {x, tokens, tokens, clusters, perm, offsets, previous, means, sums, nullptr};
    rc = launch_update_t<float>(uj, 1, batch, dims, clusters, stream);
  }
  cudaError_t f = cudaFreeAsync(scratch, stream);
  if (!rc && f != cudaSuccess) rc = static_cast<int>(f);
  return rc;
}

extern "C" int peco_kmeans_fit(const void* q_x, long long q_head_rows, int q_tokens, int q_clusters, int32_t* q_labels,
                               const float* q_init, float* q_centers, float* q_work, float* q_norms, int32_t* q_counts,
                               int32_t* q_offsets, int32_t* q_perm, const void* k_x, long long k_head_rows, int k_tokens,
                               int k_clusters, int32_t* k_labels, const float* k_init, float* k_centers, float* k_work,
                               float* k_norms, int32_t* k_counts, int32_t* k_offsets, int32_t* k_perm, int bh, int dims,
                               int iters, void* stream) {
  KmeansProblem p[2];
  p[0] = {q_x, q_head_rows, q_tokens, q_clusters, q_init, q_work, q_centers, q_norms, q_labels, q_counts, q_offsets, q_perm};
  p[1] = {k_x, k_head_rows, k_tokens, k_clusters, k_init, k_work, k_centers, k_norms, k_labels, k_counts, k_offsets, k_perm};
  const int njobs = k_x ? 2 : 1;
  return kmeans_fit_bf16(njobs, p, bh, dims, iters, static_cast<cudaStream_t>(stream));
}
