// Cluster-pair selection (peco/clustering.py:139-186) and the text partition
// extension (peco/processor.py:68-84).  Two kernels: a register-tiled fp32
// score GEMM writes every (query, key cluster) logit to stream-ordered
// scratch; then one CTA per query cluster does the softmax, the sort and the
// keep rule.
//
// Per query cluster g of a head:
//   s_c   = (Cq[g] . Ck[c]) * fp32(D^-0.5)
//   l_c   = s_c + log(count_c)            (-inf for empty key clusters)
//   p_c   = exp(l_c - max l) / max(sum exp, FLT_MIN)
//   order = stable sort of p descending   (ties keep the lower index first)
//   keep  = (mass before < top_p) | first | position < ceil(min_ratio*CK)
//   map   = keep & count_k > 0 & count_q > 0
// The running mass is accumulated in double and rounded to fp32 per element,
// as torch's CPU cumsum does.  Results agree with the fp32 CPU reference up to
// ulp-level ties of p (scores use a different summation order).
#include <float.h>

#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

constexpr int kTile = 64;        // score tile: 64 query x 64 key clusters
constexpr int kRowThreads = 256;  // row kernel: one CTA per query cluster

__device__ __forceinline__ unsigned long long sort_key(float p, int idx) {
  // p >= 0: its bit pattern orders like the value; invert for descending.
  return (static_cast<unsigned long long>(~__float_as_uint(p)) << 32) | static_cast<unsigned>(idx);
}

// logits[h, g, c] = (Cq[h,g] . Ck[h,c]) * fp32(D^-0.5) + log(count_c), -inf for
// empty key clusters.  Each dot product is one fmaf chain in ascending d.
// grid (ceil(CK/64), ceil(CQ/64), BH), 256 threads, each a 4x4 output block;
// smem holds both tiles transposed ([d][row]) so a thread's 4 rows are one
// float4.
template <int D>
__global__ void __launch_bounds__(256) select_scores_kernel(const float* __restrict__ qc, const float* __restrict__ kc,
                                                            const int32_t* __restrict__ k_sizes,
                                                            float* __restrict__ logits, int cq, int ck) {
  extern __shared__ __align__(16) float ssm[];
  float* qt = ssm;               // [D][64]
  float* kt = ssm + D * kTile;   // [D][64]
  const int head = blockIdx.z;
  const int g0 = blockIdx.y * kTile, c0 = blockIdx.x * kTile;
  const float* qh = qc + static_cast<long long>(head) * cq * D;
  const float* kh = kc + static_cast<long long>(head) * ck * D;
  // consecutive threads take consecutive rows, so the transposed stores hit
  // consecutive shared-memory words (no bank conflicts)
  for (int i = threadIdx.x; i < kTile * D / 4; i += blockDim.x) {
    const int row = i % kTile, d4 = (i / kTile) * 4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (g0 + row < cq) a = *reinterpret_cast<const float4*>(qh + static_cast<long long>(g0 + row) * D + d4);
    if (c0 + row < ck) b = *reinterpret_cast<const float4*>(kh + static_cast<long long>(c0 + row) * D + d4);
    qt[(d4 + 0) * kTile + row] = a.x;
    qt[(d4 + 1) * kTile + row] = a.y;
    qt[(d4 + 2) * kTile + row] = a.z;
    qt[(d4 + 3) * kTile + row] = a.w;
    kt[(d4 + 0) * kTile + row] = b.x;
    kt[(d4 + 1) * kTile + row] = b.y;
    kt[(d4 + 2) * kTile + row] = b.z;
    kt[(d4 + 3) * kTile + row] = b.w;
  }
  __syncthreads();
  const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
#pragma unroll 8
  for (int d = 0; d < D; ++d) {
    const float4 qa = *reinterpret_cast<const float4*>(qt + d * kTile + 4 * ty);
    const float4 kb = *reinterpret_cast<const float4*>(kt + d * kTile + 4 * tx);
    const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(qv[a], kv[b], acc[a][b]);
  }
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(D)));
  const int32_t* ks = k_sizes + static_cast<long long>(head) * ck;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int g = g0 + 4 * ty + a;
    if (g >= cq) continue;
    float* out = logits + (static_cast<long long>(head) * cq + g) * ck;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int c = c0 + 4 * tx + b;
      if (c >= ck) continue;
      const int n = ks[c];
      out[c] = n > 0 ? acc[a][b] * scale + logf(static_cast<float>(n)) : -INFINITY;
    }
  }
}

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = is_max ? -INFINITY : 0.0f;
  for (int w = 0; w < nw; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  return r;
}
// One CTA per (query cluster, head): softmax of the logits row, stable
// descending sort of (p, index), running mass in double rounded to fp32 per
// element, keep rule, map row.  smem: sort keys [np2] u64 | p [np2] f32.
__global__ void __launch_bounds__(kRowThreads) select_row_kernel(const float* __restrict__ logits,
                                                                 const int32_t* __restrict__ q_sizes,
                                                                 const int32_t* __restrict__ k_sizes,
                                                                 uint8_t* __restrict__ map, int cq, int ck, int np2,
                                                                 float top_p, int minimum, int extend, int out_cols) {
  extern __shared__ __align__(16) unsigned char rsm[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(rsm);
  float* e = reinterpret_cast<float*>(keys + np2);
  __shared__ float red[32];
  __shared__ double dscan[32];
  const int g = blockIdx.x, head = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row_in = logits + (static_cast<long long>(head) * cq + g) * ck;
  const int32_t* ks = k_sizes + static_cast<long long>(head) * ck;
  float mx = -INFINITY;
  for (int c = tid; c < ck; c += blockDim.x) {
    const float l = row_in[c];
    e[c] = l;
    mx = fmaxf(mx, l);
  }
  mx = block_reduce(mx, true, red);
  if (!isfinite(mx)) mx = 0.0f;
  float sum = 0.0f;
  for (int c = tid; c < ck; c += blockDim.x) {
    const float v = expf(e[c] - mx);
    e[c] = v;
    sum += v;
  }
  sum = fmaxf(block_reduce(sum, false, red), FLT_MIN);
  for (int c = tid; c < np2; c += blockDim.x) keys[c] = c < ck ? sort_key(e[c] / sum, c) : ~0ull;
  __syncthreads();
  // bitonic sort ascending on keys (descending p, ascending index)
  for (int k = 2; k <= np2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = keys[i], b = keys[l];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            keys[i] = b;
            keys[l] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // running mass in double, per-element fp32 rounding; each thread owns a
  // contiguous span of sorted positions
  const int per = (ck + blockDim.x - 1) / blockDim.x;
  const int p0 = min(ck, tid * per), p1 = min(ck, p0 + per);
  double local = 0.0;
  for (int i = p0; i < p1; ++i) local += static_cast<double>(__uint_as_float(~static_cast<unsigned>(keys[i] >> 32)));
  double incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) dscan[warp] = incl;
  __syncthreads();
  double carry = 0.0;
  for (int w = 0; w < warp; ++w) carry += dscan[w];
  double run = carry + incl - local;
  const int qn = q_sizes[static_cast<long long>(head) * cq + g];
  uint8_t* row = map + (static_cast<long long>(head) * (extend ? cq + 2 : cq) + g) * out_cols;
  for (int i = p0; i < p1; ++i) {
    const unsigned long long key = keys[i];
    const float p = __uint_as_float(~static_cast<unsigned>(key >> 32));
    const int c = static_cast<int>(key & 0xffffffffu);
    run += static_cast<double>(p);
    const float before = __fsub_rn(static_cast<float>(run), p);
    bool keep = (before < top_p) || (top_p >= 1.0f) || (i == 0) || (i < minimum);
    keep = keep && ks[c] > 0 && qn > 0;
    row[c] = keep ? 1 : 0;
  }
  if (extend && tid == 0) {
    row[ck] = 1;      // every video query sees the valid text keys
    row[ck + 1] = 0;  // ... never the padding keys
  }
}

// Text rows of the extended map and the extended size vectors of one head,
// by the threads first, first + step, ... (a block or a warp).
__device__ __forceinline__ void write_text_partition(int head, int first, int step, uint8_t* __restrict__ map,
                                                     const int32_t* __restrict__ q_sizes,
                                                     const int32_t* __restrict__ k_sizes, int32_t* __restrict__ q_ext,
                                                     int32_t* __restrict__ k_ext, int cq, int ck, int valid_text,
                                                     int text_length) {
  const int cols = ck + 2;
  uint8_t* base = map + static_cast<long long>(head) * (cq + 2) * cols;
  for (int c = first; c < cols; c += step) {
    base[static_cast<long long>(cq) * cols + c] = c < cols - 1 ? 1 : 0;       // valid text row
    base[static_cast<long long>(cq + 1) * cols + c] = c == cols - 1 ? 1 : 0;  // padding row
  }
  for (int c = first; c < cq; c += step) q_ext[static_cast<long long>(head) * (cq + 2) + c] = q_sizes[static_cast<long long>(head) * cq + c];
  for (int c = first; c < ck; c += step) k_ext[static_cast<long long>(head) * (ck + 2) + c] = k_sizes[static_cast<long long>(head) * ck + c];
  if (first == 0) {
    q_ext[static_cast<long long>(head) * (cq + 2) + cq] = valid_text;
    q_ext[static_cast<long long>(head) * (cq + 2) + cq + 1] = text_length - valid_text;
    k_ext[static_cast<long long>(head) * (ck + 2) + ck] = valid_text;
    k_ext[static_cast<long long>(head) * (ck + 2) + ck + 1] = text_length - valid_text;
  }
}

// The same row computation with one WARP per (query cluster, head) for up to
// 256 key clusters: element i = r * 32 + lane lives in register r of a lane,
// so the bitonic sort runs on shuffles (partner lanes) and register swaps
// (partner registers) with no block barrier, and the running mass is NPL
// warp scans.  Sums use a different order than the CTA kernel (per-lane
// partials, then a butterfly), so p can differ from it in the last ulp.
template <int NPL>  // keys per lane: np2 = 32 * NPL
__global__ void __launch_bounds__(256) select_row_warp_kernel(const float* __restrict__ logits,
                                                              const int32_t* __restrict__ q_sizes,
                                                              const int32_t* __restrict__ k_sizes,
                                                              uint8_t* __restrict__ map, int cq, int ck, float top_p,
                                                              int minimum, int extend, int out_cols, int rows,
                                                              int32_t* __restrict__ q_ext, int32_t* __restrict__ k_ext,
                                                              int valid_text, int text_length) {
  const int wid = static_cast<int>((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= rows) return;
  const int head = wid / cq, g = wid - head * cq;
  const float* row_in = logits + (static_cast<long long>(head) * cq + g) * ck;
  const int32_t* ks = k_sizes + static_cast<long long>(head) * ck;
  float e[NPL];
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < NPL; ++r) {
    const int c = r * 32 + lane;
    e[r] = c < ck ? row_in[c] : -INFINITY;
    mx = fmaxf(mx, e[r]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (!isfinite(mx)) mx = 0.0f;
  float sum = 0.0f;
#pragma unroll
  for (int r = 0; r < NPL; ++r) {
    const int c = r * 32 + lane;
    e[r] = c < ck ? expf(e[r] - mx) : 0.0f;
    sum += e[r];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  sum = fmaxf(sum, FLT_MIN);
  unsigned long long key[NPL];
#pragma unroll
  for (int r = 0; r < NPL; ++r) {
    const int c = r * 32 + lane;
    key[r] = c < ck ? sort_key(e[r] / sum, c) : ~0ull;
  }
  // bitonic sort, ascending keys (descending p, ascending index)
#pragma unroll
  for (int k = 2; k <= 32 * NPL; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {  // partner in this lane: register r ^ (j / 32)
        const int jr = j >> 5;
#pragma unroll
        for (int r = 0; r < NPL; ++r) {
          const int pr = r ^ jr;
          if (pr > r) {
            const int i = r * 32 + lane;
            const bool up = (i & k) == 0;
            const unsigned long long a = key[r], b = key[pr];
            if ((a > b) == up) {
              key[r] = b;
              key[pr] = a;
            }
          }
        }
      } else {  // partner lane ^ j, same register
#pragma unroll
        for (int r = 0; r < NPL; ++r) {
          const int i = r * 32 + lane;
          const bool up = (i & k) == 0, lower = (lane & j) == 0;
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, key[r], j);
          const unsigned long long lo = key[r] < other ? key[r] : other, hi = key[r] < other ? other : key[r];
          key[r] = (lower == up) ? lo : hi;
        }
      }
    }
  }
  // running mass over sorted positions i = r * 32 + lane, in double
  const int qn = q_sizes[static_cast<long long>(head) * cq + g];
  uint8_t* row = map + (static_cast<long long>(head) * (extend ? cq + 2 : cq) + g) * out_cols;
  double carry = 0.0;
#pragma unroll
  for (int r = 0; r < NPL; ++r) {
    const int i = r * 32 + lane;
    const float p = i < ck ? __uint_as_float(~static_cast<unsigned>(key[r] >> 32)) : 0.0f;
    double incl = static_cast<double>(p);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const double run = carry + incl;
    carry += __shfl_sync(0xffffffffu, incl, 31);
    if (i < ck) {
      const int c = static_cast<int>(key[r] & 0xffffffffu);
      const float before = __fsub_rn(static_cast<float>(run), p);
      bool keep = (before < top_p) || (top_p >= 1.0f) || (i == 0) || (i < minimum);
      keep = keep && ks[c] > 0 && qn > 0;
      row[c] = keep ? 1 : 0;
    }
  }
  if (extend && lane == 0) {
    row[ck] = 1;      // every video query sees the valid text keys
    row[ck + 1] = 0;  // ... never the padding keys
  }
  // the warp of query cluster 0 also writes its head's text partition (one
  // launch less than a kernel of its own)
  if (extend && g == 0)
    write_text_partition(head, lane, 32, map, q_sizes, k_sizes, q_ext, k_ext, cq, ck, valid_text, text_length);
}

__global__ void text_partition_kernel(uint8_t* __restrict__ map, const int32_t* __restrict__ q_sizes,
                                      const int32_t* __restrict__ k_sizes, int32_t* __restrict__ q_ext,
                                      int32_t* __restrict__ k_ext, int cq, int ck, int valid_text, int text_length) {
  write_text_partition(blockIdx.x, threadIdx.x, blockDim.x, map, q_sizes, k_sizes, q_ext, k_ext, cq, ck, valid_text,
                       text_length);
}

}  // namespace

int launch_select(const float* qc, const float* kc, const int32_t* qs, const int32_t* ks, uint8_t* map, int bh,
                  int cq, int ck, int dims, float top_p, int minimum, int extend, int valid_text, int text_length,
                  int32_t* q_ext, int32_t* k_ext, float* logits_in, cudaStream_t stream) {
  if (bh < 1 || bh > 65535 || cq < 1 || ck < 1 || cq > 65535) return kErrInvalidValue;
  if (dims != 64 && dims != 128) return kErrUnsupported;
  if ((reinterpret_cast<uintptr_t>(qc) | reinterpret_cast<uintptr_t>(kc)) & 15) return kErrInvalidValue;
  int np2 = 1;
  while (np2 < ck) np2 <<= 1;
  const size_t row_smem = (sizeof(unsigned long long) + sizeof(float)) * static_cast<size_t>(np2);
  if (row_smem > 200 * 1024) return kErrUnsupported;
  // logits in the caller's buffer, else in stream-ordered scratch of this call
  void* scratch = nullptr;
  cudaError_t e = cudaSuccess;
  if (!logits_in) {
    e = cudaMallocAsync(&scratch, sizeof(float) * static_cast<size_t>(bh) * cq * ck, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  float* logits = logits_in ? logits_in : static_cast<float*>(scratch);
  const size_t tile_smem = sizeof(float) * 2 * kTile * dims;
  dim3 sgrid((ck + kTile - 1) / kTile, (cq + kTile - 1) / kTile, bh);
  int rc = 0;
  if (dims == 128) {
    e = cudaFuncSetAttribute(select_scores_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(tile_smem));
    if (e == cudaSuccess) select_scores_kernel<128><<<sgrid, 256, tile_smem, stream>>>(qc, kc, ks, logits, cq, ck);
  } else {
    e = cudaFuncSetAttribute(select_scores_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(tile_smem));
    if (e == cudaSuccess) select_scores_kernel<64><<<sgrid, 256, tile_smem, stream>>>(qc, kc, ks, logits, cq, ck);
  }
  rc = e != cudaSuccess ? static_cast<int>(e) : launch_status();
  if (!rc && row_smem > 48 * 1024) {
    e = cudaFuncSetAttribute(select_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(row_smem));
    if (e != cudaSuccess) rc = static_cast<int>(e);
  }
  if (!rc) {
    const int out_cols = extend ? ck + 2 : ck;
    const int rows = bh * cq;
    const int wgrid = (rows + 7) / 8;  // 8 warps (rows) per block
    if (np2 <= 32) {
      select_row_warp_kernel<1><<<wgrid, 256, 0, stream>>>(logits, qs, ks, map, cq, ck, top_p, minimum, extend, out_cols, rows,
                                                            q_ext, k_ext, valid_text, text_length);
    } else if (np2 == 64) {
      select_row_warp_kernel<2><<<wgrid, 256, 0, stream>>>(logits, qs, ks, map, cq, ck, top_p, minimum, extend, out_cols, rows,
                                                            q_ext, k_ext, valid_text, text_length);
    } else if (np2 == 128) {
      select_row_warp_kernel<4><<<wgrid, 256, 0, stream>>>(logits, qs, ks, map, cq, ck, top_p, minimum, extend, out_cols, rows,
                                                            q_ext, k_ext, valid_text, text_length);
    } else if (np2 == 256) {
      select_row_warp_kernel<8><<<wgrid, 256, 0, stream>>>(logits, qs, ks, map, cq, ck, top_p, minimum, extend, out_cols, rows,
                                                            q_ext, k_ext, valid_text, text_length);
    } else {
      select_row_kernel<<<dim3(cq, bh), kRowThreads, row_smem, stream>>>(logits, qs, ks, map, cq, ck, np2, top_p,
                                                                         minimum, extend, out_cols);
    }
    rc = launch_status();
  }
  if (scratch) {
    e = cudaFreeAsync(scratch, stream);
    if (!rc && e != cudaSuccess) rc = static_cast<int>(e);
  }
  if (rc || !extend || np2 <= 256) return rc;  // the warp kernel wrote the text partition
  text_partition_kernel<<<bh, 256, 0, stream>>>(map, qs, ks, q_ext, k_ext, cq, ck, valid_text, text_length);
  return launch_status();
}

}  // namespace peco

extern "C" int peco_select_cluster_connections(const float* q_centroids, const float* k_centroids,
                                               const int32_t* q_sizes, const int32_t* k_sizes, uint8_t* map,
                                               int bh, int cq, int ck, int dims, float top_p, int minimum,
                                               float* logits, void* stream) {
  if (!(top_p >= 0.0f && top_p <= 1.0f) || minimum < 0) return peco::kErrInvalidValue;
  return peco::launch_select(q_centroids, k_centroids, q_sizes, k_sizes, map, bh, cq, ck, dims, top_p, minimum, 0,
                             0, 0, nullptr, nullptr, logits, static_cast<cudaStream_t>(stream));
}

extern "C" int peco_select_text_partition(const float* q_centroids, const float* k_centroids,
                                          const int32_t* q_sizes, const int32_t* k_sizes, uint8_t* map_ext,
                                          int32_t* q_sizes_ext, int32_t* k_sizes_ext, int bh, int cq, int ck,
                                          int dims, float top_p, int minimum, int valid_text, int text_length,
                                          float* logits, void* stream) {
  if (!(top_p >= 0.0f && top_p <= 1.0f) || minimum < 0 || valid_text < 0 || valid_text > text_length)
    return peco::kErrInvalidValue;
  return peco::launch_select(q_centroids, k_centroids, q_sizes, k_sizes, map_ext, bh, cq, ck, dims, top_p, minimum, 1,
                             valid_text, text_length, q_sizes_ext, k_sizes_ext, logits,
                             static_cast<cudaStream_t>(stream));
}
