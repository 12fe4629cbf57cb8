/*
 * C ABI of libpeco_b200.so -- the B200-native (sm_100a) PECO attention hot path.
 *
 * Plain pointers and sizes only.  Every function enqueues work on the CUDA
 * stream passed as the last argument (a cudaStream_t as void*), never
 * synchronises, and returns 0 on success, a cudaError_t value for CUDA
 * failures, or one of the PECO_ERR_* codes below.  Buffers are allocated by
 * the caller (the reference's convention, peco/clustering_cuda.py:83-90 and
 * peco/attention_cuda.py:128); the exceptions are three drop-in symbols whose
 * reference signatures pass no room for what the sm_100a kernels need:
 * peco_assign_tokens_to_centers (bf16 split of fp32 tokens and centres),
 * peco_recompute_cluster_centers (sort scratch) and peco_sparse_attention
 * (attention plan and key blocks) take it from the stream-ordered allocator
 * (cudaMallocAsync / cudaFreeAsync on the caller's stream), as do the two
 * selection entry points for their [BH,CQ,CK] fp32 logits.
 *
 * Device-side faults are never raised with traps: kernels skip out-of-range
 * indices and give up bounded waits, OR-ing a bit into a per-device status
 * word that peco_device_status() returns.
 *
 * Citations are to the reference project Tom-HKUST/PECO.
 */
#ifndef PECO_B200_H_
#define PECO_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PECO_ERR_UNSUPPORTED 20001  /* shape or dtype outside the kernels' support */
#define PECO_ERR_TENSOR_MAP 20002   /* TMA descriptor could not be encoded */
#define PECO_ERR_DRIVER 20003       /* driver entry point unavailable */
#define PECO_ERR_TIMEOUT 20004      /* a device-side bounded wait expired */
#define PECO_ERR_WORKSPACE 20005    /* workspace too small */
#define PECO_ERR_CAPACITY 20006     /* problem larger than a no-alloc entry point's fixed scratch */

#define PECO_STATUS_TIMEOUT 1u      /* status word bit: a bounded wait expired */
#define PECO_STATUS_BAD_INDEX 2u    /* status word bit: an index failed its bounds check */

/* ---- drop-in symbols (same signatures and status conventions) ---------- */

/* Nearest-centre labels for fp32 x [B,N,D] and centres [B,C,D]; writes
 * labels [B,N] and center_norms [B,C] = ||c||^2.  ``scratch`` ([chunk,C] in
 * the reference) is accepted and left untouched.  D in {64,128}.
 * Replaces peco/kernels/kmeans.cu:139-175 (bound at peco/clustering_cuda.py:65,93-108). */
int peco_assign_tokens_to_centers(const float* x, const float* centers, int32_t* labels, float* scratch,
                                  float* center_norms, int batch, int tokens, int dims, int clusters,
                                  int chunk_size, void* stream);

/* means[b,c] = mean of the tokens labelled c (empty -> previous), counts,
 * and sums.  Deterministic (no atomics).
 * Replaces peco/kernels/kmeans.cu:179-196 (bound at peco/clustering_cuda.py:66,111-125). */
int peco_recompute_cluster_centers(const float* x, const int32_t* labels, const float* previous, float* sums,
                                   int32_t* counts, float* means, int batch, int tokens, int dims, int clusters,
                                   void* stream);

/* Row permutation of [B*H,N,D] items of 2 or 4 bytes: forward
 * out[j] = in[idx[j]], inverse out[idx[j]] = in[j]; bit-exact copies.
 * Replaces peco/kernels/kmeans.cu:200-217 (bound at peco/clustering_cuda.py:67,128-146). */
int peco_reorder_token_features(const void* input, const int32_t* indices, void* output, int batch_heads,
                                int tokens, int dims, int item_size, int inverse, void* stream);

/* peco_recompute_cluster_centers without any allocation (no counterpart in
 * the reference): identical results, with the sort scratch -- batch*tokens +
 * batch*(clusters+1) ints -- in a fixed per-device array of
 * peco_recompute_cluster_centers_static_capacity() ints (2^21, 8 MiB); larger
 * problems return PECO_ERR_CAPACITY without launching.  For callers that must
 * not allocate once running: a serving loop that pre-plans all its memory
 * (an allocation can fail or stall under fragmentation there), or a process
 * whose stream-ordered pool is unavailable or capped.  The first call on a
 * device looks up the array's address (cudaGetSymbolAddress) and should come
 * before any stream capture; the address is kept for the process's lifetime,
 * so do not call it on a device after cudaDeviceReset there (the array, and
 * the address, are gone with the context).  Nothing in the scratch must
 * start at zero.
 * Calls that overlap on one device share the scratch and race; serialise
 * them. */
int peco_recompute_cluster_centers_static(const float* x, const int32_t* labels, const float* previous,
                                          float* sums, int32_t* counts, float* means, int batch, int tokens,
                                          int dims, int clusters, void* stream);
long long peco_recompute_cluster_centers_static_capacity(void);

/* Error text for the clustering entry points (peco/kernels/kmeans.cu:220-223). */
const char* peco_cluster_error_message(int code);

/* Cluster-masked softmax(QK^T/sqrt(D))V over group-packed Q [BH,SQ,D] and
 * K/V [BH,SK,D]; map [BH,CQ,CK] bytes, sizes int32 [BH,CQ]/[BH,CK]; rows with
 * no allowed key -> 0.  dtype 0 = fp16, 1 = bf16; D in {64,128}.  Workspace:
 * int32 BH*(CK+2+3*(ceil(SQ/16)+CQ)) (the reference's size), accepted for
 * ABI compatibility: the plan and key blocks (peco_attention_plan,
 * peco_pack_key_blocks) live in stream-ordered scratch of the call.
 * Replaces peco/kernels/sparse_attention.cu:210-230 (bound at peco/attention_cuda.py:57,130-137). */
int peco_sparse_attention(const void* q, const void* k, const void* v, const uint8_t* selected,
                          const int* q_sizes, const int* k_sizes, void* output, int* workspace, int bh, int sq,
                          int sk, int d, int cq, int ck, int dtype, void* stream);

/* Error text for the attention entry point (peco/kernels/sparse_attention.cu:232-234). */
const char* peco_attention_error_string(int code);

/* ---- fused entry points (used by the processor's fast path) ------------ */

/* Stable argsort of labels [rows,N] (values in [0,C)) by counting sort:
 * indices [rows,N] (original token at each packed position), counts
 * [rows,C] and offsets [rows,C+1] (either may be NULL).
 * Replaces torch.argsort(stable=True) at peco/clustering.py:105. */
int peco_sort_labels(const int32_t* labels, int32_t* indices, int32_t* counts, int32_t* offsets, int rows,
                     int tokens, int clusters, void* stream);

/* Fixed-iteration Lloyd k-means of bf16 token rows for up to two problems
 * (Q and K of one call) in the same launches.  Head b of problem x starts at
 * row b*head_rows (so the video prefix of a [BH,S,D] tensor needs no copy).
 * Per problem: init [BH,C,D] fp32 (read), centers (final means of the last
 * partition, may alias init), work (BH * peco_kmeans_work_floats(C, D, N)
 * floats: ping-pong centres, the centres' bf16 tensor-core image, the
 * token norms the first iteration records for the rest and, for long
 * sequences, the label sort's per-segment scratch), norms [BH,C],
 * labels [BH,N], counts [BH,C], offsets [BH,C+1], perm [BH,N] (stable
 * argsort of the final labels).  Pass k_x = NULL for a single problem.
 * Replaces fit_token_clusters' CUDA loop, peco/clustering.py:59-88 with tol=0. */
int peco_kmeans_fit(const void* q_x, long long q_head_rows, int q_tokens, int q_clusters, int32_t* q_labels,
                    const float* q_init, float* q_centers, float* q_work, float* q_norms, int32_t* q_counts,
                    int32_t* q_offsets, int32_t* q_perm, const void* k_x, long long k_head_rows, int k_tokens,
                    int k_clusters, int32_t* k_labels, const float* k_init, float* k_centers, float* k_work,
                    float* k_norms, int32_t* k_counts, int32_t* k_offsets, int32_t* k_perm, int bh, int dims,
                    int iters, void* stream);

/* Floats of ``work`` per head for peco_kmeans_fit (-1 for unsupported sizes). */
long long peco_kmeans_work_floats(int clusters, int dims, int tokens);

/* Boolean map [BH,CQ,CK] of kept (query cluster, key cluster) pairs: stable
 * descending sort of softmax(Cq.Ck^T/sqrt(D) + log count_k), keep while the
 * mass before < top_p (all if top_p == 1), the first, and the first
 * ``minimum``; AND nonempty.  ``logits``: fp32 [BH,CQ,CK] scratch of the
 * caller, or null for stream-ordered scratch of the call.  Replaces
 * peco/clustering.py:139-186. */
int peco_select_cluster_connections(const float* q_centroids, const float* k_centroids, const int32_t* q_sizes,
                                    const int32_t* k_sizes, uint8_t* map, int bh, int cq, int ck, int dims,
                                    float top_p, int minimum, float* logits, void* stream);

/* Same selection written straight into the text-extended map
 * [BH,CQ+2,CK+2] with extended sizes [BH,CQ+2]/[BH,CK+2].
 * Replaces peco/clustering.py:154-186 followed by peco/processor.py:68-84. */
int peco_select_text_partition(const float* q_centroids, const float* k_centroids, const int32_t* q_sizes,
                               const int32_t* k_sizes, uint8_t* map_ext, int32_t* q_sizes_ext,
                               int32_t* k_sizes_ext, int bh, int cq, int ck, int dims, float top_p, int minimum,
                               int valid_text, int text_length, float* logits, void* stream);

/* Base-Offset PE over [BH,N,D] (dtype 0 fp16, 1 bf16, 2 fp32; D in {64,128};
 * bits 4 or 8).  mode 0: out = fake-quantized x; mode 1: codes uint8
 * [BH,N,D], offset_min / scale fp32 [BH,N]; mode 2: out = decode(codes).
 * Bit-exact with peco/quantization.py:96-150. */
int peco_base_offset(int mode, const void* x, const int32_t* labels, const float* centroids, void* out,
                     uint8_t* codes, float* offset_min, float* scale, int bh, int tokens, int dims, int clusters,
                     int bits, int dtype, void* stream);

/* Attention plan (workspace: int32 bh * peco_attention_workspace_stride),
 * from the group map [BH,GQ,GK] and sizes [BH,GQ]/[BH,GK] (extents clamped
 * like peco/kernels/sparse_attention.cu:25-31): the work units (<= 128 query
 * rows of one query group), the key-row -> key-block map and, per unit, the
 * selected key clusters.  Key blocks hold K or V as 8-row blocks of 8*D
 * 16-bit elements in the tensor core's shared-memory image (D/64 panels of
 * 8 rows x 128 bytes, 16-byte chunk c of row i at chunk c^i); each key
 * cluster starts a new block.  When k_blocks/v_blocks ([BH,
 * peco_key_block_rows(sk, gk), D]) are given, the padding rows of every
 * cluster's last block are zeroed.  Splits the planning half of
 * peco/kernels/sparse_attention.cu:17-52 out of the attention launch. */
int peco_attention_plan(const uint8_t* map, const int* q_sizes, const int* k_sizes, void* k_blocks,
                        void* v_blocks, int* workspace, int bh, int sq, int sk, int d, int gq, int gk,
                        void* stream);

long long peco_attention_workspace_stride(int sq, int sk, int gq, int gk);
long long peco_key_block_rows(int sk, int gk);

/* Row-major K/V [BH,SK,D] -> key blocks through a plan.  Used by the drop-in
 * peco_sparse_attention (which plans and packs internally). */
int peco_pack_key_blocks(const void* k, const void* v, void* k_blocks, void* v_blocks, const int* workspace,
                         int bh, int sq, int sk, int d, int gq, int gk, void* stream);

/* One pass over bf16 Q/K/V [BH,S,D] (video tokens first): packed row j of
 * each head takes source video row indices[j] -- Base-Offset fake quantized
 * for Q and K when bits > 0, copied for V (which uses K's indices) -- and
 * text rows j >= video are copied in place.  With ``plan`` (a workspace
 * written by peco_attention_plan with sq = sk = seq), K and V rows go to
 * key blocks (k_packed/v_packed [BH, peco_key_block_rows(seq, gk), D])
 * instead of row-major [BH,S,D].  Replaces peco/processor.py:141-149 (fake
 * quant, three gathers and the concats). */
int peco_quantize_gather(const void* q, const void* k, const void* v, void* q_packed, void* k_packed,
                         void* v_packed, const int32_t* q_indices, const int32_t* k_indices,
                         const int32_t* q_labels, const int32_t* k_labels, const float* q_centroids,
                         const float* k_centroids, int q_clusters, int k_clusters, int bh, int seq, int video,
                         int dims, int bits, const int* plan, int gq, int gk, void* stream);

/* Sparse attention of packed bf16 Q [BH,SQ,D] over key blocks, following a
 * plan from peco_attention_plan; output rows are scattered through the
 * inverse permutation: packed row j < video goes to row q_indices[j] of
 * ``output`` (q_indices null: no scatter), text rows stay in place.
 * Fuses peco/kernels/sparse_attention.cu with peco/clustering.py:127-136. */
int peco_sparse_attention_restore(const void* q, const void* k_blocks, const void* v_blocks,
                                  const int* workspace, void* output, int bh, int sq, int sk, int d, int gq,
                                  int gk, const int32_t* q_indices, int video, void* stream);

/* Input stage of the attention processor: from the bf16 projection outputs
 * of the video rows (vq/vk/vv) and the text rows (tq/tk/tv), each a
 * row-major [rows, H*D] view with ``*_stride`` elements between rows, write
 * bf16 Q/K/V [H, video_rows + text_rows, D] (video rows first).  Per (row,
 * head): Q and K are RMS-normalised with the stream's gains (w*_v / w*_t,
 * fp32 [D]; null: no norm), rounded to bf16, and video rows are rotated with
 * the (cos, sin) tables [video_rows, D] fp32, pairs interleaved (null: no
 * rotation); V is copied.  Replaces the head split, norm_q/norm_k,
 * apply_rotary_emb, concatenations and contiguous copies of
 * peco/processor.py:163-188. */
int peco_prepare_qkv(const void* vq, const void* vk, const void* vv, long long v_stride, int video_rows,
                     const void* tq, const void* tk, const void* tv, long long t_stride, int text_rows,
                     const float* wq_v, const float* wk_v, float eps_v, const float* wq_t, const float* wk_t,
                     float eps_t, const float* cos, const float* sin, void* q, void* k, void* v, int heads,
                     int dims, void* stream);

/* Sequence <-> head reshard of sequence-sharded attention over NVLink peer
 * memory (no counterpart in the reference, which runs on one GPU; it replaces
 * the NCCL all-to-all of the long-video configuration).  ``buffers`` and
 * ``flags`` are device arrays of every rank's receive buffer and flag array
 * (int64 [slots][world]) as mapped in this process (torch symmetric memory).
 * peco_exchange_put copies ``pieces`` contiguous blocks of ``piece_bytes``
 * (16-byte multiple) from src + src_offsets[i] to rank dst_ranks[i]'s buffer
 * + dst_offsets[i] with plain stores, then sets this rank's entry of slot
 * ``flag_slot`` in every rank's flag array to ``epoch``; ``done_counter`` is a
 * zeroed device unsigned the launch uses and resets.  peco_exchange_wait
 * makes ``stream`` wait until every rank's entry of the slot in this rank's
 * flag array has reached ``epoch`` (bounded: on expiry the device status word
 * records a timeout). */
int peco_exchange_put(const void* src, const long long* src_offsets, const int* dst_ranks,
                      const long long* dst_offsets, long long piece_bytes, int pieces,
                      const unsigned long long* buffers, const unsigned long long* flags, int flag_slot,
                      int rank, int world, long long epoch, unsigned* done_counter, void* stream);
int peco_exchange_wait(const long long* flags, int world, int flag_slot, long long epoch, void* stream);

/* ---- diagnostics --------------------------------------------------------- */

/* Copies the device status word of the current device to *out (synchronising
 * ``stream``) and clears it when ``clear`` != 0. */
int peco_device_status(unsigned* out, int clear, void* stream);

const char* peco_error_string(int code);

int peco_library_version(void);

/* Number of kernels this library has launched in the process so far. */
unsigned long long peco_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif  /* PECO_B200_H_ */
