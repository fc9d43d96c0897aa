// augur_decode.cu — one layer of a batch's decode step behind one C call.
//
// augur runs its paged attention branch one sequence at a time
// (augur/attention.py:53-86, batch 1 per augur/paged_kv_cache.py:179-180).
// For a decode step of a whole batch the KV-cache side of a layer is two
// launches here: the fused RoPE write of the new tokens, then decode
// attention over every cached sequence. augur_kv_decode_layer issues both
// from a per-step argument block, so a caller's per-layer cost is one foreign
// call with the layer's own tensors (the host side of a decode step is what
// bounds it at small batches).

#include <stdint.h>

#include "augur_kv.h"
#include "common.cuh"

using augur_kv_dev::elem_size;
using augur_kv_dev::fail;

#define AUGUR_KV_EXPORT extern "C" __attribute__((visibility("default")))

AUGUR_KV_EXPORT int augur_kv_decode_layer(augur_kv_decode_args* A, int32_t layer, const void* q,
                                          const void* key, const void* value, void* out, void* stream) {
  if (A == nullptr) return fail(AUGUR_KV_EINVAL, "decode_layer: null args");
  if (layer < 0 || layer >= A->n_layers)
    return fail(AUGUR_KV_EINVAL, "decode_layer: layer %d outside [0, %d)", layer, A->n_layers);
  const int es = elem_size(A->dtype);
  if (es == 0) return fail(AUGUR_KV_EINVAL, "decode_layer: unknown dtype %d", A->dtype);
  if (A->k_pool == nullptr || A->v_pool == nullptr)
    return fail(AUGUR_KV_EINVAL, "decode_layer: null pool");
  const int64_t layer_bytes = int64_t(layer) * A->pool_strides[0] * es;
  char* kl = static_cast<char*>(A->k_pool) + layer_bytes;
  char* vl = static_cast<char*>(A->v_pool) + layer_bytes;
  const int Hq = A->n_q_heads, D = A->head_dim;
  // token b of the step is (row 0, column b): source element (b, h, d) at
  // base + b*strides[2] + h*strides[3] + d; destination (block, row, head)
  const int64_t kv_src[4] = {0, 0, A->kv_strides[0], A->kv_strides[1]};
  const int64_t q_src[4] = {0, 0, A->q_strides[0], A->q_strides[1]};
  const int64_t q_rot[4] = {0, 0, int64_t(Hq) * D, D};
  const int64_t dst[4] = {0, A->pool_strides[1], A->pool_strides[3], A->pool_strides[2]};
  const int64_t col[2] = {0, 1};
  const int64_t dense[2] = {int64_t(Hq) * D, D};
  const int64_t pool[3] = {A->pool_strides[1], A->pool_strides[2], A->pool_strides[3]};
  // One launch: the attention kernel rotates q and the new k itself and
  // writes the new k and v to their pool rows (position seq_lens[b] - 1 and
  // its slot in the block table; positions[b] and slots[b] must name the
  // same, as DecodeStep and DecodeGraphStep build them, and the kernel
  // records AUGUR_KV_EBOUNDS where they do not).
  const augur_kv_dev::FusedRope fr{key,         value,       A->kv_strides[0], A->kv_strides[1],
                                   A->rope_cos, A->rope_sin, A->rope_positions, A->positions,
                                   A->slots};
  const int64_t q_two[2] = {A->q_strides[0], A->q_strides[1]};
  bool fused = false;
  int rc = augur_kv_dev::paged_decode_attention_impl(
      q, q_two, kl, vl, pool, A->num_blocks, A->block_size, A->block_tables, A->tables_stride, A->max_blocks,
      A->seq_lens, A->max_seq_len, A->batch, Hq, A->n_kv_heads, D, A->dtype, out, dense, A->flags, A->counters,
      A->counters_bytes, A->scratch, A->scratch_bytes, A->status, stream, &fr, &fused);
  A->launches = fused ? 1 : 0;
  if (rc != AUGUR_KV_OK || fused) return rc;
  A->launches = 2;
  // otherwise the RoPE write, then the attention
  rc = augur_kv_rope_scatter(key, value, kv_src, kv_src, A->batch, A->dtype, kl, vl, dst, A->block_size,
                                 A->num_blocks, A->slots, col, 0, A->positions, col, A->rope_cos, A->rope_sin,
                                 A->rope_positions, q, q_src, A->q_rot, q_rot, Hq, A->batch, 1, A->n_kv_heads, D,
                                 A->status, stream);
  if (rc != AUGUR_KV_OK) return rc;
  // the RoPE write just ahead of it writes the new tokens' pool rows: no early reads
  return augur_kv_paged_decode_attention(A->q_rot, dense, kl, vl, pool, A->num_blocks, A->block_size,
                                         A->block_tables, A->tables_stride, A->max_blocks, A->seq_lens,
                                         A->max_seq_len, A->batch, Hq, A->n_kv_heads, D, A->dtype, out, dense,
                                         A->flags & ~AUGUR_KV_ATTN_EARLY_READS, A->counters, A->counters_bytes, A->scratch, A->scratch_bytes,
                                         A->status, stream);
}
