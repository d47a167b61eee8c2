// Multi-head latent attention for one decode token (mla.cu).
#pragma once
#include "common.cuh"

namespace moe {

struct MlaDims {
  int64_t heads;  // num_heads
  int64_t L;      // cache positions attended (the new one included)
  int64_t nope;   // qk_nope_dim
  int64_t rope;   // qk_rope_dim
  int64_t R;      // kv_lora_rank
  int64_t v;      // v_head_dim
};

constexpr int64_t kMlaMaxLatent = 1024;  // kv_lora_rank (4 latent columns per attention thread)
constexpr int64_t kMlaMaxRope = 256;
constexpr int64_t kMlaMaxNope = 8192;

// kOk when the kernels take these (already positive / non-negative) dimensions.
int mla_supported(const MlaDims& d);
// Workspace of the attention core (absorbed queries, rotated q_pe, per-split partials).
int64_t mla_core_workspace_bytes(const MlaDims& d);
// Workspace of the whole block (the core plus q_low, the kv_a row, q and the head outputs).
int64_t mla_block_workspace_bytes(const MlaDims& d, int64_t q_rank);

// The attention core: q_nope[h] at q_nope + h * nope_stride, q_pe[h] at q_pe +
// h * pe_stride (rotated here by cos/sin when given), caches [L, R] / [L, rope],
// wkv_b [heads, nope + v, R] -> out [heads, v].  Device pointers, fp32.
int mla_core_run(const MlaDims& d, const float* q_nope, int64_t nope_stride, const float* q_pe, int64_t pe_stride,
                 const float* rope_cos, const float* rope_sin, const float* kv_cache, const float* pe_cache,
                 const float* wkv_b, float* out, float softmax_scale, char* workspace, cudaStream_t stream);

struct MlaBlockArgs {
  const float* hidden;       // [H]
  const float* q_a;          // [q_rank, H]
  const float* q_b;          // [heads * (nope + rope), q_rank]
  const float* kv_a;         // [R + rope, H]
  const float* kv_b;         // [heads * (nope + v), R]
  const float* o_w;          // [H, heads * v]
  const float* q_norm;       // [q_rank]
  const float* kv_norm;      // [R]
  const float* prev_kv;      // [prev_len, R] or null when prev_len == 0
  const float* prev_pe;      // [prev_len, rope]
  const float* rope_cos;     // [rope / 2]
  const float* rope_sin;
  float* next_kv;            // [prev_len + 1, R]
  float* next_pe;            // [prev_len + 1, rope]
  float* out;                // [H]
  int64_t H, q_rank, prev_len;
  float eps, softmax_scale;
};
// The block (d.L = prev_len + 1).
int mla_block_run(const MlaDims& d, const MlaBlockArgs& a, char* workspace, cudaStream_t stream);

}  // namespace moe
