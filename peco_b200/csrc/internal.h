// Declarations shared between the library's translation units (not part of
// the public C ABI in include/peco_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace peco {

// One fixed-iteration k-means problem on bf16 token rows.
struct KmeansProblem {
  const void* x;          // bf16 rows; head b starts at row b * head_rows
  long long head_rows;
  int tokens;             // tokens per head
  int clusters;
  const float* centers_a; // initial centres [B, C, D] (may alias centers_out or centers_b)
  float* centers_b;       // ping-pong buffer [B, C, D]
  float* centers_out;     // final centres (means of the last partition)
  float* norms;           // [B, C] scratch: squared centre norms
  int32_t* labels;        // [B, tokens] labels of the last assignment
  int32_t* counts;        // [B, C] sizes of the last partition
  int32_t* offsets;       // [B, C+1] cluster starts in the packed order
  int32_t* perm;          // [B, tokens] stable argsort of the last labels
};

int kmeans_fit_bf16(int njobs, const KmeansProblem* probs, int bh, int dims, int iters, cudaStream_t stream);

int launch_stable_sort(const int32_t* labels, long long label_stride, int rows, int tokens, int clusters,
                       int32_t* indices, int32_t* counts, int32_t* offsets, cudaStream_t stream);

int launch_select(const float* qc, const float* kc, const int32_t* qs, const int32_t* ks, uint8_t* map, int bh,
                  int cq, int ck, int dims, float top_p, int minimum, int extend, int valid_text, int text_length,
                  int32_t* q_ext, int32_t* k_ext, cudaStream_t stream);

int launch_quant_gather(const void* q, const void* k, const void* v, void* qp, void* kp, void* vp,
                        const int32_t* q_perm, const int32_t* k_perm, const int32_t* q_labels,
                        const int32_t* k_labels, const float* q_cen, const float* k_cen, int cq, int ck, int bh,
                        int seq, int video, int dims, int bits, cudaStream_t stream);

int launch_sparse_attention(const void* q, const void* k, const void* v, const uint8_t* map, const int* q_sizes,
                            const int* k_sizes, void* out, int* ws, int ws_stride, int bh, int sq, int sk, int d,
                            int gq, int gk, int dtype, const int32_t* perm, int video, cudaStream_t stream);

long long attention_ws_stride(int sq, int gq, int gk);

}  // namespace peco
