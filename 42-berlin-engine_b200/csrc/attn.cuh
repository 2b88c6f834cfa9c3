// attn.cuh -- KV append, LSH index and decode attention kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace ec {

// Device layout of the decode state of one context (all sequences, layers).
struct KvLayout {
  int n_layers, n_heads, n_kv_heads, head_dim, seq_len;
  int max_blocks;       // per (sequence, layer): ceil(seq_len / 16)
  int paged;            // 1 paged INT8, 0 linear BF16
  // paged INT8: block (seq, layer, physical b) at index ((seq*L + layer)*MB + b)
  int8_t* kq;           // [S*L*MB][KV][16][hd]
  int8_t* vq;
  float* ks;            // [S*L*MB][KV][16]
  float* vs;
  float* centroid;      // [S*L*MB][hd]
  int* page_table;      // [S*L*MB] logical -> physical (within the sequence+layer)
  // linear BF16: [S*L][seq_len][KV][hd]
  uint16_t* lk;
  uint16_t* lv;
  int shared_cache;     // linear: every sequence index reads sequence 0's cache
  int seq_plus1;        // paged prefill: every batch row addresses sequence
                        // seq_plus1 - 1 (0: row b addresses sequence b)
};

// The sequence whose paged KV cache batch row b reads and writes.
inline __host__ __device__ int kv_seq(const KvLayout& kv, int b) {
  return kv.seq_plus1 ? kv.seq_plus1 - 1 : b;
}

struct LshLayout {
  int tables, bits, unit, max_units, radius, max_cand;
  const float* hp;      // [tables][bits][head_dim]
  // per sequence
  float* acc;           // [S][head_dim]
  int* meta;            // [S][4]: acc_count, acc_start, n_units, pad
  uint32_t* unit_hash;  // [S][tables][max_units]
  int* unit_start;      // [S][max_units]
  int* unit_len;        // [S][max_units]
  int* heads;           // [S][tables][1 << bits]
  int* next;            // [S][tables][max_units]
  unsigned long long* counters;  // [S][2]: sparse queries, sum of attended K
};

struct StepBuffers {
  const int* pos;       // [B]
  float* qkv;           // [B][(H + 2KV) * hd] projections (k rotated in place)
  float* qrot;          // [B][H * hd] rotated queries
  float* att;           // [B][H * hd]
  int* sel;             // [B][L?] per-sequence selection scratch: [B][max_sel]
  int* nsel;            // [B]
  int* selp;            // split attention: the selection's physical blocks [B][max_sel]
  int max_sel;
  const float* rope_cos;  // [seq_len][hd/2]
  const float* rope_sin;
  int sparse_k, window, sparse_blocks_k;
  int* err;
  int pos_fixed;        // position when pos == nullptr (per-op entry points)
  int q_rotated;        // selection reads qrot (already rotated) instead of qkv
  int list_dense;       // selection also lists every block when attending all
  // linear mode: candidates and their scores between the selection's
  // kernels ([B][linear_cand_cap] each) and the candidate count ([B])
  int* lcand;
  float* lscore;
  int* lnc;
  int defer_centroid;   // paged prefill: the append leaves block centroids to
                        // launch_paged_centroids (rows of one launch share a block)
  int fast_tpc;         // split attention: tokens per CTA (set by its launcher)
  // tensor parallelism (linear mode): the LSH query mean reads every rank's
  // rotated queries (q_all [B][h_all][hd], all-gathered), and the candidate
  // scores leave their per-KV-head dots in score_parts [B][cap][KV] for the
  // cross-rank sum in head order (tp_sum_scores)
  const float* q_all;
  int h_all;
  float* score_parts;
};

// Linear-mode candidate capacity per sequence: the window plus max_cand
// units of `unit` tokens; the selection runs as kLinearSelectLaunches kernels.
constexpr int kLinearSelectLaunches = 3;
inline __host__ __device__ int linear_cand_cap(const StepBuffers& sb, const LshLayout& lsh) {
  return sb.window + lsh.max_cand * lsh.unit;
}

inline __host__ __device__ int step_pos(const StepBuffers& sb, int b) {
  return sb.pos ? sb.pos[b] : sb.pos_fixed;
}

// Shared-memory attributes for the current device (outside stream capture).
cudaError_t attn_prepare(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb);
// Per layer, before attention: one CTA appends the token (RoPE, INT8 or BF16
// store, centroid, LSH update); in paged mode a second CTA selects the
// blocks to attend (it only reads blocks that this step does not change).
cudaError_t launch_kv_append(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                             int layer, int B, cudaStream_t s, bool pdl);
// Paged prefill: block centroids of sequence `seq`, layer `layer`, for the
// blocks whose last token lies in [first_pos, first_pos + n); then the block
// selection of every batch row (after the centroids, unlike kv_append's CTA 1).
cudaError_t launch_paged_centroids(const KvLayout& kv, int layer, int seq, int first_pos, int n,
                                   cudaStream_t s);
// Paged prefill, layer 0: the LSH index update of every batch row in row
// order (kv_append skips it when rows share a sequence).
cudaError_t launch_lsh_update_rows(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                                   int B, cudaStream_t s);
cudaError_t launch_paged_select_rows(const KvLayout& kv, const StepBuffers& sb, int layer, int B,
                                     cudaStream_t s);
cudaError_t launch_linear_select(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                                 int layer, int B, cudaStream_t s, bool pdl);
// The same in three pieces for tensor parallelism: candidates (every rank,
// identical), per-KV-head dots into sb.score_parts (this rank's heads), and,
// once the dots of all ranks are gathered ([world][cap][KV per rank] from
// `parts_all`), their sum in global head order followed by the heap.
cudaError_t launch_linear_candidates(const KvLayout& kv, const LshLayout& lsh,
                                     const StepBuffers& sb, int layer, int B, cudaStream_t s);
cudaError_t launch_linear_score_parts(const KvLayout& kv, const LshLayout& lsh,
                                      const StepBuffers& sb, int layer, int B, cudaStream_t s);
cudaError_t launch_linear_sum_heap(const LshLayout& lsh, const StepBuffers& sb,
                                   const float* parts_all, int world, int kv_local, int B,
                                   cudaStream_t s);
// lsh_update (layer 0, KV head 0) from a key vector that is not in sb.qkv
// (tensor parallelism: the gathered keys of every rank)
cudaError_t launch_lsh_update_key(const LshLayout& lsh, const StepBuffers& sb, const float* k,
                                  int hd, cudaStream_t s);
cudaError_t launch_attention(const KvLayout& kv, const StepBuffers& sb, int layer, int B,
                             cudaStream_t s, bool pdl);
// Batched paged steps whose attention runs as attention_group_kernel (one CTA
// per KV head and sequence, the reference's order): faster than the split
// attention from 4 sequences on, so split mode keeps it there.
bool use_group_attention(const KvLayout& kv, const StepBuffers& sb, int B);

// Per-op entry points on one layer (a KvLayout with n_layers = 1):
// append one token, select blocks (sb.q_rotated), attention with max_tok.
cudaError_t launch_paged_append_view(const KvLayout& kv, const float* k, const float* v, int pos,
                                     int* err, cudaStream_t s);
cudaError_t launch_paged_select(const KvLayout& kv, const StepBuffers& sb, cudaStream_t s);
cudaError_t launch_attention_n(const KvLayout& kv, const StepBuffers& sb, int max_tok,
                               cudaStream_t s);
size_t attention_smem_bytes(int max_tok, int hd, bool paged);

// Split attention (attn_fast.cu), paged KV: per layer one CTA per sequence
// appends the token and selects the top-K block set by ranks, then a
// cluster of `fast_splits` CTAs per (KV head, sequence) attends with the
// reference's softmax weights and merges over distributed shared memory.
bool fast_attention_supported(const KvLayout& kv, int sparse_blocks_k);
int fast_splits(int B);
cudaError_t fast_attention_prepare(const KvLayout& kv);
cudaError_t launch_fast_select(const KvLayout& kv, const LshLayout& lsh, const StepBuffers& sb,
                               int layer, int B, cudaStream_t s, bool pdl);
cudaError_t launch_fast_attend(const KvLayout& kv, StepBuffers sb, int layer, int B,
                               cudaStream_t s, bool pdl);

}  // namespace ec
