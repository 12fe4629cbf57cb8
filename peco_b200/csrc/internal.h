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
  unsigned char* image;   // [B, image bytes per head] bf16 hi/lo image of the centres being assigned against
  float* xnorm;           // [B, tokens] token norms |x| (written by the first assignment, read by the rest)
  int32_t* sort_seg;      // [B, sort_segments(tokens), C] sort scratch, or null (one CTA per head)
};

int kmeans_fit_bf16(int njobs, const KmeansProblem* probs, int bh, int dims, int iters, cudaStream_t stream);

int launch_stable_sort(const int32_t* labels, long long label_stride, int rows, int tokens, int clusters,
                       int32_t* indices, int32_t* counts, int32_t* offsets, cudaStream_t stream);

// One stable counting sort of labels [rows, tokens] (values in [0, clusters)).
struct SortJobInput {
  const int32_t* labels;
  long long label_stride;
  int rows, tokens, clusters;
  int32_t* indices;   // [rows, tokens]
  int32_t* counts;    // [rows, clusters] or null
  int32_t* offsets;   // [rows, clusters + 1] or null
  int32_t* seg;       // optional [rows, segs, clusters] scratch: split each row over segs CTAs
  int segs;
};

// CTAs per row for the label sort of a k-means fit (0: one CTA per row).  Long
// rows are split so that few heads still fill the GPU; their scratch is
// segs * clusters ints per row.
inline int sort_segments(int tokens) {
  if (tokens < 32768) return 0;
  const int s = (tokens + 8191) / 8192;
  return s < 16 ? s : 16;
}
int launch_stable_sort_jobs(const SortJobInput* jobs, int njobs, cudaStream_t stream);

int launch_select(const float* qc, const float* kc, const int32_t* qs, const int32_t* ks, uint8_t* map, int bh,
                  int cq, int ck, int dims, float top_p, int minimum, int extend, int valid_text, int text_length,
                  int32_t* q_ext, int32_t* k_ext, float* logits, cudaStream_t stream);

// ---------------------------------------------------------------------------
// Attention plan and key blocks
// ---------------------------------------------------------------------------
// Keys and values reach the attention kernel as 8-row KEY BLOCKS: every key
// cluster starts a new block (its last block is zero-padded), and a block
// holds the byte image the tensor core reads from shared memory -- D/64
// panels of 8 rows x 128 bytes, the 16-byte chunk c of row i stored at chunk
// position c ^ i (128-byte swizzle).  One contiguous run of blocks is then one
// bulk copy.  Head h owns blocks [h * blocks, (h + 1) * blocks).
constexpr int kKeyBlockRows = 8;
constexpr int kUnitRows = 128;  // query rows per attention work unit

// Per-head plan workspace (int32), written by the planner kernel:
//   [0] unit count, [1] split pieces, [2..3] reserved
//   kp    [gk+1]            clamped row start of every key cluster
//   gp    [gk+1]            first key block of every key cluster
//   units [max_units][8]    q_start, q_count, entry count, block count, first
//                           group, groups, group bounds, split (piece << 16 |
//                           part << 8 | parts; 0 = whole)
//   rows  [sk]              key row -> row in the key-block image (-1: unused)
//   ent   [max_units][gk]   int2 entries, one per selected key cluster:
//                           (first block - first position, end position << 4 | rows in last block)
//   ptab  [2 kSplitPieces]  q_start, q_count of every split piece
//   part  [kSplitPieces][kSplitParts][kUnitRows][kPartCols] floats: the split
//         parts' unnormalised outputs, then [..][kUnitRows][2]: their max and sum
// The last int of the last head's region is the work counter of the
// persistent attention kernel.
// ints per work unit in the plan: q_start, q_count, entries, blocks, first
// query group, groups, group bounds, split
constexpr int kUnitInts = 8;

// Calls with few heads split the key range of their first large query group
// (the text rows, which attend every key) over kSplitParts units, so that
// group's long key walk runs on several CTAs; a combine kernel merges the
// parts' partial softmax results.
constexpr int kSplitPieces = 4;    // 128-row pieces of that group that may split
constexpr int kSplitParts = 4;     // key-range parts per piece
constexpr int kPartCols = 128;     // partial output columns (D <= 128)
// Split only short sequences: there the text units' key walk is about twice
// a CTA's average share at <= 4 heads; at 119k keys it is barely above it and
// the four parts' separate streams over the keys cost more L2 reuse than the
// balance gains (measured: +5.6% attention at 3 heads).
inline int attention_split_parts(int bh, int sk) { return bh <= 4 && sk <= 32768 ? kSplitParts : 1; }

struct PlanGeom {
  int sq, sk, gq, gk;
  long long max_units, blocks;
  long long off_kp, off_gp, off_units, off_rows, off_ent, off_ptab, off_part, off_ml, stride;
};

__host__ __device__ inline PlanGeom plan_geom(int sq, int sk, int gq, int gk) {
  PlanGeom g;
  g.sq = sq;
  g.sk = sk;
  g.gq = gq;
  g.gk = gk;
  g.max_units = (static_cast<long long>(sq) + kUnitRows - 1) / kUnitRows + gq + kSplitPieces * (kSplitParts - 1);
  g.blocks = (static_cast<long long>(sk) + kKeyBlockRows - 1) / kKeyBlockRows + gk;
  g.off_kp = 4;
  g.off_gp = g.off_kp + gk + 1;
  g.off_units = (g.off_gp + gk + 1 + 3) & ~3LL;
  g.off_rows = g.off_units + kUnitInts * g.max_units;
  g.off_ent = (g.off_rows + sk + 3) & ~3LL;
  g.off_ptab = (g.off_ent + 2 * g.max_units * gk + 3) & ~3LL;
  g.off_part = g.off_ptab + 2 * kSplitPieces;
  g.off_ml = g.off_part + static_cast<long long>(kSplitPieces) * kSplitParts * kUnitRows * kPartCols;
  g.stride = (g.off_ml + 2LL * kSplitPieces * kSplitParts * kUnitRows + 1 + 3) & ~3LL;
  return g;
}

// byte offset of element (row i, dim d) inside one key block (2-byte elements)
__host__ __device__ inline int key_block_offset(int i, int d) {
  return (d >> 6) * 1024 + i * 128 + ((((d & 63) >> 3) ^ i) << 4) + (d & 7) * 2;
}

int launch_quant_gather(const void* q, const void* k, const void* v, void* qp, void* kp, void* vp,
                        const int32_t* q_perm, const int32_t* k_perm, const int32_t* q_labels,
                        const int32_t* k_labels, const float* q_cen, const float* k_cen, int cq, int ck, int bh,
                        int seq, int video, int dims, int bits, const int* plan, int gq, int gk,
                        cudaStream_t stream);

int launch_attention_plan(const uint8_t* map, const int* q_sizes, const int* k_sizes, void* k_blocks,
                          void* v_blocks, int* ws, int bh, int sq, int sk, int d, int gq, int gk,
                          cudaStream_t stream);

int launch_pack_key_blocks(const void* k, const void* v, void* k_blocks, void* v_blocks, const int* ws, int bh,
                           int sq, int sk, int d, int gq, int gk, cudaStream_t stream);

int launch_attention_main(const void* q, const void* k_blocks, const void* v_blocks, const int* ws, void* out,
                          int bh, int sq, int sk, int d, int gq, int gk, int dtype, const int32_t* perm, int video,
                          cudaStream_t stream);

}  // namespace peco
