// Input stage of the attention processor (peco/processor.py:159-188): from
// the projection outputs to the [H, S, D] Q/K/V of one PECO call in a single
// pass over HBM.
//
// The reference splits heads with a view, normalises Q and K per head with
// the attention module's RMSNorm, applies the rotary embedding to the video
// rows, concatenates the text rows and makes every tensor contiguous -- a
// dozen elementwise kernels and copies per tensor.  Here one warp takes one
// (row, head) pair: it reads the head's D elements of Q, K and V once (8 or 4
// bytes per lane), normalises Q and K, rotates the video rows and writes the
// three rows to their place in the head-major output.
//
// Numerics (bf16 in and out, fp32 inside): RMSNorm is x * rsqrt(mean(x^2) +
// eps) * w with each product rounded to fp32 and the result rounded once to
// bf16; the rotation is (x * cos) + (x_rot * sin) on the bf16 normalised
// value, pairs interleaved (x_rot[2i] = -x[2i+1], x_rot[2i+1] = x[2i]), each
// product and the sum rounded to fp32, then to bf16.  Only the order of the
// D-term sum of squares differs from a torch evaluation of the same formula.
#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {
namespace {

struct PrepareArgs {
  const __nv_bfloat16* src[2][3];  // [stream: video, text][q, k, v]
  long long stride[2];             // elements between consecutive rows of a stream
  int rows[2];
  const float* wq[2];              // RMSNorm gains [D] per stream (null: no norm)
  const float* wk[2];
  float eps[2];
  const float* cos;                // [video rows, D] (null: no rotation)
  const float* sin;
  __nv_bfloat16* dst[3];           // [H, S, D]
  int heads;
  unsigned* status;
};

template <int E>
struct Vec;
template <>
struct Vec<4> {
  using T = uint2;
};
template <>
struct Vec<2> {
  using T = uint32_t;
};

template <int E>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&x)[E]) {
  const typename Vec<E>::T u = *reinterpret_cast<const typename Vec<E>::T*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < E / 2; ++e) {
    const float2 f = __bfloat1622float2(h[e]);
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
}

template <int E>
__device__ __forceinline__ void store_row(__nv_bfloat16* p, const float (&x)[E]) {
  typename Vec<E>::T u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < E / 2; ++e) h[e] = __floats2bfloat162_rn(x[2 * e], x[2 * e + 1]);
  *reinterpret_cast<typename Vec<E>::T*>(p) = u;
}

// RMS normalisation of one head row held E elements per lane (dims lane*E..)
template <int D, int E>
__device__ __forceinline__ void rms_norm(float (&x)[E], const float* w, float eps, int lane) {
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
  const float mean = __fmul_rn(warp_sum(ss), 1.0f / D);
  const float r = rsqrtf(__fadd_rn(mean, eps));
#pragma unroll
  for (int e = 0; e < E; ++e) {
    x[e] = __fmul_rn(__fmul_rn(x[e], r), w[lane * E + e]);
    x[e] = __bfloat162float(__float2bfloat16_rn(x[e]));  // the norm's output is a bf16 tensor
  }
}

template <int D, int E>
__device__ __forceinline__ void rotate(float (&x)[E], const float* c, const float* s, int lane) {
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    const int d = lane * E + e;
    const float a = x[e], b = x[e + 1];
    x[e] = __fadd_rn(__fmul_rn(a, c[d]), __fmul_rn(-b, s[d]));
    x[e + 1] = __fadd_rn(__fmul_rn(b, c[d + 1]), __fmul_rn(a, s[d + 1]));
  }
}

// One warp per (row, head); rows of both streams in one index space, heads
// fastest so that consecutive warps read consecutive memory.
template <int D>
__global__ void __launch_bounds__(256) prepare_qkv_kernel(const PrepareArgs a) {
  constexpr int E = D / 32;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(a.rows[0] + a.rows[1]) * a.heads;
  const long long s_all = a.rows[0] + a.rows[1];
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long w = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
       w += warps) {
    const long long row = w / a.heads;
    const int h = static_cast<int>(w - row * a.heads);
    const int st = row < a.rows[0] ? 0 : 1;
    const long long r = st ? row - a.rows[0] : row;
    const long long in_off = r * a.stride[st] + static_cast<long long>(h) * D + lane * E;
    const long long out_off = (static_cast<long long>(h) * s_all + row) * D + lane * E;
    float x[E];
    // Q and K: norm, then the rotation on video rows
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      load_row<E>(a.src[st][t] + in_off, x);
      const float* wgt = t == 0 ? a.wq[st] : a.wk[st];
      if (wgt) rms_norm<D, E>(x, wgt, a.eps[st], lane);
      if (st == 0 && a.cos) rotate<D, E>(x, a.cos + r * D, a.sin + r * D, lane);
      store_row<E>(a.dst[t] + out_off, x);
    }
    // V: moved as is
    *reinterpret_cast<typename Vec<E>::T*>(a.dst[2] + out_off) =
        *reinterpret_cast<const typename Vec<E>::T*>(a.src[st][2] + in_off);
  }
}

}  // namespace
}  // namespace peco

using namespace peco;

extern "C" int peco_prepare_qkv(const void* vq, const void* vk, const void* vv, long long v_stride, int video_rows,
                                const void* tq, const void* tk, const void* tv, long long t_stride, int text_rows,
                                const float* wq_v, const float* wk_v, float eps_v, const float* wq_t,
                                const float* wk_t, float eps_t, const float* cos, const float* sin, void* q, void* k,
                                void* v, int heads, int dims, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (dims != 64 && dims != 128) return kErrUnsupported;
  if (heads < 1 || video_rows < 0 || text_rows < 0 || video_rows + text_rows < 1) return kErrInvalidValue;
  if (!vq || !vk || !vv || !q || !k || !v || (text_rows > 0 && (!tq || !tk || !tv))) return kErrInvalidValue;
  if ((cos == nullptr) != (sin == nullptr)) return kErrInvalidValue;
  const long long row_elems = static_cast<long long>(heads) * dims;
  if (v_stride < row_elems || (text_rows > 0 && t_stride < row_elems)) return kErrInvalidValue;
  // every lane moves D/32 two-byte elements with one aligned access
  const int align = dims == 128 ? 8 : 4;
  auto misaligned = [&](const void* p) { return p && (reinterpret_cast<uintptr_t>(p) % align) != 0; };
  if (misaligned(vq) || misaligned(vk) || misaligned(vv) || misaligned(tq) || misaligned(tk) || misaligned(tv) ||
      misaligned(q) || misaligned(k) || misaligned(v) || (v_stride * 2) % align || (t_stride * 2) % align)
    return kErrInvalidValue;
  PrepareArgs a{};
  const void* src[2][3] = {{vq, vk, vv}, {tq, tk, tv}};
  for (int s = 0; s < 2; ++s)
    for (int t = 0; t < 3; ++t) a.src[s][t] = static_cast<const __nv_bfloat16*>(src[s][t]);
  a.stride[0] = v_stride;
  a.stride[1] = t_stride;
  a.rows[0] = video_rows;
  a.rows[1] = text_rows;
  a.wq[0] = wq_v;
  a.wk[0] = wk_v;
  a.wq[1] = wq_t;
  a.wk[1] = wk_t;
  a.eps[0] = eps_v;
  a.eps[1] = eps_t;
  a.cos = cos;
  a.sin = sin;
  a.dst[0] = static_cast<__nv_bfloat16*>(q);
  a.dst[1] = static_cast<__nv_bfloat16*>(k);
  a.dst[2] = static_cast<__nv_bfloat16*>(v);
  a.heads = heads;
  a.status = device_status_ptr();
  const long long warps = static_cast<long long>(video_rows + text_rows) * heads;
  // 8 warps per block and at most 8 blocks per SM (a full SM of warps), each
  // warp striding over the (row, head) pairs beyond one grid
  const long long want = (warps + 7) / 8;
  const int grid = static_cast<int>(want < 148LL * 8 ? want : 148LL * 8);
  if (dims == 128) prepare_qkv_kernel<128><<<grid, 256, 0, stream>>>(a);
  else prepare_qkv_kernel<64><<<grid, 256, 0, stream>>>(a);
  return launch_status();
}
