// Cluster-pair selection (peco/clustering.py:139-186) and the text partition
// extension (peco/processor.py:68-84), one warp per query cluster.
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

constexpr int kSelWarps = 8;
constexpr int kKeyChunk = 32;

__device__ __forceinline__ unsigned long long sort_key(float p, int idx) {
  // p >= 0: its bit pattern orders like the value; invert for descending.
  return (static_cast<unsigned long long>(~__float_as_uint(p)) << 32) | static_cast<unsigned>(idx);
}

// grid: (ceil(CQ / W), BH); block: 32 * W (W <= kSelWarps warps, one per query cluster).
// smem: sort keys [W][np2] u64 | probabilities [W][np2] f32 | q rows [W][D] f32 |
//       key chunk [kKeyChunk][D+1] f32
__global__ void __launch_bounds__(32 * kSelWarps) select_kernel(
    const float* __restrict__ qc, const float* __restrict__ kc, const int32_t* __restrict__ q_sizes,
    const int32_t* __restrict__ k_sizes, uint8_t* __restrict__ map, int cq, int ck, int dims, int np2, float top_p,
    int minimum, int extend, int out_cols) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nwarps = blockDim.x >> 5;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem);       // [W][np2]
  float* probs = reinterpret_cast<float*>(keys + static_cast<long long>(nwarps) * np2);  // [W][np2]
  float* qrow = probs + static_cast<long long>(nwarps) * np2;                  // [W][D]
  float* kchunk = qrow + nwarps * dims;                                        // [kKeyChunk][D+1]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int g = blockIdx.x * nwarps + warp;
  const bool active = g < cq;
  const float* qh = qc + (static_cast<long long>(head) * cq) * dims;
  const float* kh = kc + (static_cast<long long>(head) * ck) * dims;
  const int32_t* ks = k_sizes + static_cast<long long>(head) * ck;
  unsigned long long* mykeys = keys + static_cast<long long>(warp) * np2;
  if (active)
    for (int d = lane; d < dims; d += 32) qrow[warp * dims + d] = qh[static_cast<long long>(g) * dims + d];
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(dims)));
  float* logit = probs + static_cast<long long>(warp) * np2;
  for (int c0 = 0; c0 < ck; c0 += kKeyChunk) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKeyChunk * dims; i += blockDim.x) {
      const int r = i / dims, d = i - r * dims;
      kchunk[r * (dims + 1) + d] = (c0 + r < ck) ? kh[static_cast<long long>(c0 + r) * dims + d] : 0.0f;
    }
    __syncthreads();
    const int c = c0 + lane;
    if (active && c < ck) {
      float s = 0.0f;
      const float* kr = kchunk + lane * (dims + 1);
      const float* qr = qrow + warp * dims;
      for (int d = 0; d < dims; ++d) s = fmaf(qr[d], kr[d], s);
      s = s * scale;
      const int n = ks[c];
      logit[c] = n > 0 ? s + logf(static_cast<float>(n)) : -INFINITY;
    }
  }
  __syncwarp();
  if (!active) return;
  float mx = -INFINITY;
  for (int c = lane; c < ck; c += 32) mx = fmaxf(mx, logit[c]);
  mx = warp_max(mx);
  if (!isfinite(mx)) mx = 0.0f;
  float sum = 0.0f;
  for (int c = lane; c < ck; c += 32) {
    const float e = expf(logit[c] - mx);
    logit[c] = e;
    sum += e;
  }
  sum = fmaxf(warp_sum(sum), FLT_MIN);
  __syncwarp();
  for (int c = lane; c < np2; c += 32) mykeys[c] = c < ck ? sort_key(logit[c] / sum, c) : ~0ull;
  __syncwarp();
  // bitonic sort ascending on keys (descending p, ascending index)
  for (int k = 2; k <= np2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < np2; i += 32) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = mykeys[i], b = mykeys[l];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            mykeys[i] = b;
            mykeys[l] = a;
          }
        }
      }
      __syncwarp();
    }
  }
  // running mass in double, per-element fp32 rounding; each lane owns a
  // contiguous span of positions
  const int per = (ck + 31) / 32;
  const int p0 = lane * per, p1 = min(ck, p0 + per);
  double local = 0.0;
  for (int i = p0; i < p1; ++i) local += static_cast<double>(__uint_as_float(~static_cast<unsigned>(mykeys[i] >> 32)));
  double incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  double run = incl - local;
  const int qn = q_sizes[static_cast<long long>(head) * cq + g];
  uint8_t* row = map + (static_cast<long long>(head) * (extend ? cq + 2 : cq) + g) * out_cols;
  for (int i = p0; i < p1; ++i) {
    const unsigned long long key = mykeys[i];
    const float p = __uint_as_float(~static_cast<unsigned>(key >> 32));
    const int c = static_cast<int>(key & 0xffffffffu);
    run += static_cast<double>(p);
    const float before = __fsub_rn(static_cast<float>(run), p);
    bool keep = (before < top_p) || (top_p >= 1.0f) || (i == 0) || (i < minimum);
    keep = keep && ks[c] > 0 && qn > 0;
    row[c] = keep ? 1 : 0;
  }
  if (extend && lane == 0) {
    row[ck] = 1;      // every video query sees the valid text keys
    row[ck + 1] = 0;  // ... never the padding keys
  }
}

// Text rows of the extended map and the extended size vectors.
__global__ void text_partition_kernel(uint8_t* __restrict__ map, const int32_t* __restrict__ q_sizes,
                                      const int32_t* __restrict__ k_sizes, int32_t* __restrict__ q_ext,
                                      int32_t* __restrict__ k_ext, int cq, int ck, int valid_text, int text_length) {
  const int head = blockIdx.x;
  const int cols = ck + 2;
  uint8_t* base = map + static_cast<long long>(head) * (cq + 2) * cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    base[static_cast<long long>(cq) * cols + c] = c < cols - 1 ? 1 : 0;       // valid text row
    base[static_cast<long long>(cq + 1) * cols + c] = c == cols - 1 ? 1 : 0;  // padding row
  }
  for (int c = threadIdx.x; c < cq; c += blockDim.x) q_ext[static_cast<long long>(head) * (cq + 2) + c] = q_sizes[static_cast<long long>(head) * cq + c];
  for (int c = threadIdx.x; c < ck; c += blockDim.x) k_ext[static_cast<long long>(head) * (ck + 2) + c] = k_sizes[static_cast<long long>(head) * ck + c];
  if (threadIdx.x == 0) {
    q_ext[static_cast<long long>(head) * (cq + 2) + cq] = valid_text;
    q_ext[static_cast<long long>(head) * (cq + 2) + cq + 1] = text_length - valid_text;
    k_ext[static_cast<long long>(head) * (ck + 2) + ck] = valid_text;
    k_ext[static_cast<long long>(head) * (ck + 2) + ck + 1] = text_length - valid_text;
  }
}

}  // namespace

int launch_select(const float* qc, const float* kc, const int32_t* qs, const int32_t* ks, uint8_t* map, int bh,
                  int cq, int ck, int dims, float top_p, int minimum, int extend, int valid_text, int text_length,
                  int32_t* q_ext, int32_t* k_ext, cudaStream_t stream) {
  if (bh < 1 || cq < 1 || ck < 1 || dims < 1 || dims > 256) return kErrInvalidValue;
  int np2 = 1;
  while (np2 < ck) np2 <<= 1;
  int warps = kSelWarps;
  auto bytes = [&](int w) {
    return (sizeof(unsigned long long) + sizeof(float)) * static_cast<size_t>(w) * np2 +
           sizeof(float) * (static_cast<size_t>(w) * dims + kKeyChunk * (dims + 1));
  };
  while (warps > 1 && bytes(warps) > 200 * 1024) --warps;
  const size_t smem = bytes(warps);
  if (smem > 220 * 1024) return kErrUnsupported;
  cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  dim3 grid((cq + warps - 1) / warps, bh);
  const int out_cols = extend ? ck + 2 : ck;
  select_kernel<<<grid, 32 * warps, smem, stream>>>(qc, kc, qs, ks, map, cq, ck, dims, np2, top_p, minimum,
                                                         extend, out_cols);
  int rc = launch_status();
  if (rc || !extend) return rc;
  text_partition_kernel<<<bh, 256, 0, stream>>>(map, qs, ks, q_ext, k_ext, cq, ck, valid_text, text_length);
  return launch_status();
}

}  // namespace peco

extern "C" int peco_select_cluster_connections(const float* q_centroids, const float* k_centroids,
                                               const int32_t* q_sizes, const int32_t* k_sizes, uint8_t* map,
                                               int bh, int cq, int ck, int dims, float top_p, int minimum,
                                               void* stream) {
  if (!(top_p >= 0.0f && top_p <= 1.0f) || minimum < 0) return peco::kErrInvalidValue;
  return peco::launch_select(q_centroids, k_centroids, q_sizes, k_sizes, map, bh, cq, ck, dims, top_p, minimum, 0,
                             0, 0, nullptr, nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int peco_select_text_partition(const float* q_centroids, const float* k_centroids,
                                          const int32_t* q_sizes, const int32_t* k_sizes, uint8_t* map_ext,
                                          int32_t* q_sizes_ext, int32_t* k_sizes_ext, int bh, int cq, int ck,
                                          int dims, float top_p, int minimum, int valid_text, int text_length,
                                          void* stream) {
  if (!(top_p >= 0.0f && top_p <= 1.0f) || minimum < 0 || valid_text < 0 || valid_text > text_length)
    return peco::kErrInvalidValue;
  return peco::launch_select(q_centroids, k_centroids, q_sizes, k_sizes, map_ext, bh, cq, ck, dims, top_p, minimum, 1,
                             valid_text, text_length, q_sizes_ext, k_sizes_ext, static_cast<cudaStream_t>(stream));
}
