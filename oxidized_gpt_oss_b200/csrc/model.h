// model.h — host-side launchers of the transformer kernels around the MoE
// block (model.cu). Internal to the library.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace oxg {

// Residual update fused with the RMS norm, one row per CTA (see model.cu).
struct NormArgs {
  float *res = nullptr;             // [rows, H] f32 residual stream (updated in place)
  int rows = 0, H = 0;
  const int32_t *tokens = nullptr;  // embedding mode: token ids [rows]
  const uint16_t *embed = nullptr;  // [V, H] bf16
  int V = 0;
  const float *add = nullptr;       // add mode: S partial arrays, add_stride floats apart
  int S = 1;
  size_t add_stride = 0;
  const uint16_t *add_bias = nullptr;  // [H] bf16 or null
  const uint16_t *gamma = nullptr;     // [H] bf16
  float eps = 1e-5f;
  uint16_t *out = nullptr;          // [rows, H] bf16
  int *err = nullptr;               // receives 60 on a token id outside [0, V)
};
cudaError_t launch_residual_norm(const NormArgs &a, cudaStream_t stream);

// Linear layer out[s][t][n] = sum_{k in split s} x[t][k] W[n][k] (bf16 in,
// f32 out). K must be a multiple of 64, x rows 16-byte aligned (ldx % 8 == 0).
// linear_splits picks the K split for a batch: enough CTAs for 2 per SM, at
// most max_rows / padded(T) splits (the partial buffer's capacity).
int linear_splits(int N, int K, int T, int n_sms, int max_rows);

// Greedy choice fused into a linear layer's epilogue (T <= 8, one split):
// per token the largest output and its row (ties to the larger row), through
// 64-bit atomicMax keys; the last CTA writes next[t] (if not null) and, with
// state_mode 1, advances the decode state {pos, step, token} (out_seq[step] =
// token) or, with state_mode 2, sets it to {set_pos, 0, token of row T-1}.
// keys [T] and count must start at zero; the last CTA leaves them so.
struct ArgmaxEpilogue {
  unsigned long long *keys = nullptr;
  unsigned int *count = nullptr;
  int32_t *next = nullptr, *state = nullptr, *out_seq = nullptr;
  int state_mode = 0, set_pos = 0;
};
cudaError_t launch_linear(const uint16_t *x, int T, int ldx, const uint16_t *W, int N, int K, int splits,
                          float *out, cudaStream_t stream, const ArgmaxEpilogue *am = nullptr);

// Paged KV cache: each kv head's cache is a pool of kv_rows rows in pages of
// 64; pages [B, max_pages] (device) gives the pool page of page p of
// sequence s (positions 64p .. 64p + 63), filled by the host as sequences
// grow. Every kernel below addresses cache rows through it.
constexpr int kKvPageRows = 64;

// q/k/v epilogue: bias, RoPE (tables [positions, 32] of cos and sin), bf16 q
// [T, nh * 64] and the K/V cache rows (pools of kv_rows rows per kv head) of
// positions pos0 + t of sequence seq. pos_dev, when not null, replaces pos0
// by the position held on the device. tok_pos / tok_seq (device, [T]), when
// not null, make token t one of its own sequence: position tok_pos[t] of
// sequence tok_seq[t].
cudaError_t launch_qkv_post(const float *part, int S, int T, int nh, int nkv, const uint16_t *bias,
                            const float *rope_cos, const float *rope_sin, int pos0, const int32_t *pos_dev,
                            int kv_rows, const int32_t *pages, int max_pages, int seq, uint16_t *q_out,
                            uint16_t *kc, uint16_t *vc, cudaStream_t stream, const int32_t *tok_pos = nullptr,
                            const int32_t *tok_seq = nullptr);

struct AttnArgs {
  const uint16_t *q = nullptr;   // [T, nh * 64] bf16
  const uint16_t *kc = nullptr, *vc = nullptr;  // [nkv, max_seq, 64] bf16 (max_seq: pool rows per kv head)
  int T = 0, nh = 0, nkv = 0, max_seq = 0, pos0 = 0;
  int split_rows = 0;            // positions of one sequence (0: max_seq); sizes the decode grid
  const int32_t *pages = nullptr;  // page table [B, max_pages] (see kKvPageRows)
  int max_pages = 0;
  int seq = 0;                   // the sequence of a one-sequence call (no tok_pos)
  const int32_t *tok_pos = nullptr, *tok_seq = nullptr;  // [T] device: one query of each of T sequences
  int max_splits = 0;            // with tok_pos: 64-key page splits of the longest sequence's full span
  int window = 0;                // > 0: keys p - window + 1 .. p
  float scale = 0.125f;
  const uint16_t *sinks = nullptr;  // [nh] bf16 or null
  float *part = nullptr;         // decode split partials (attn_part_floats per query token)
  const int32_t *pos_dev = nullptr;  // T == 1: the query position read on the device (graph replays)
  uint16_t *out = nullptr;       // [T, nh * 64] bf16
  // with tok_pos and G = 8: the tensor-core decode kernel, which loads K / V
  // tiles through kv_map (a CUtensorMap over the whole KV cache, make_kv_map);
  // k_row / v_row are the map rows of this layer's K and V caches (kv head 0,
  // cache row 0)
  const void *kv_map = nullptr;
  long long k_row = 0, v_row = 0;
  int n_sms = 0;
  int *err = nullptr;            // timeout code of the tensor-core decode kernel
  // tensor-core kernel: per (token, kv head) arrival counters [T * nkv], zero
  // between launches; the last split to finish merges the splits and the sink
  // (null: attn_combine_kernel merges them — for large batches, where the
  // fence before each split's arrival stalls the warps' TMA streams)
  unsigned *merge_cnt = nullptr;
};
// A 2-D tensor map over the KV cache `kv` of `rows` rows of 64 bf16 (128-byte
// swizzle, 64-row boxes) into map (128 bytes, 64-byte aligned); rows < 2^31.
cudaError_t make_kv_map(void *map, const uint16_t *kv, long long rows);
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t stream);
size_t attn_part_floats(int nkv, int G, int max_seq);
// Page splits (64 keys each) the keys lo .. hi of a query touch.
inline int attn_page_splits(int lo, int hi) { return (hi >> 6) - (lo >> 6) + 1; }
int attn_max_group();

// next[row] = greedy choice (next may be null). With state (one row): the
// decode-step bookkeeping {position, step, token}: out_seq[step] = token,
// state token = token, position and step advance by one.
cudaError_t launch_argmax(const float *logits, int rows, int V, int32_t *next, int32_t *state, int32_t *out_seq,
                          cudaStream_t stream);
// state = {pos, 0, *tok}
cudaError_t launch_set_state(int32_t *state, int pos, const int32_t *tok, cudaStream_t stream);

}  // namespace oxg
