/*
 * augur_kv.h — C ABI of libaugur_kv.so, the sm_100a data-movement layer for
 * augur's KV caches (contiguous cache, paged cache, prefix cache).
 *
 * Every entry point takes raw device pointers, element strides as int64 host
 * arrays, int32/int64 device index arrays and the caller's cudaStream_t (as
 * void*). Nothing here allocates, synchronises or keeps state between calls
 * except the thread-local text returned by augur_kv_last_error(). All work is
 * stream-ordered on the given stream. A call with no work (zero tokens, runs
 * or layers) returns AUGUR_KV_OK without looking at its data pointers, which
 * may then be NULL (torch gives empty tensors a NULL data pointer).
 * Validation that needs host data (shapes, position ranges, allocator
 * state) is the host wrapper's job; the kernels
 * still bounds-check every index they dereference and, instead of touching
 * memory out of range, record AUGUR_KV_EBOUNDS in the optional device status
 * word (int32, first error wins) and skip that row.
 *
 * Layout vocabulary (reference shapes, augur/kv_cache.py:27-33 and
 * augur/paged_kv_cache.py:152-158):
 *   contiguous cache  [layers, batch, kv_heads, max_seq, head_dim]
 *   paged pool        [layers, num_blocks, kv_heads, block_size, head_dim]
 * A "row" is head_dim contiguous elements of one (layer, token, head) of K or
 * V. A "slot" addresses one token position of a cache: slot = major *
 * rows_per_major + row, where major is the block id (paged pool) or the batch
 * row (contiguous cache, rows_per_major = max_seq).
 */
#ifndef AUGUR_KV_H
#define AUGUR_KV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point and written to status words. */
#define AUGUR_KV_OK 0
#define AUGUR_KV_EINVAL 1   /* bad argument: null pointer, size, dtype, stride, alignment */
#define AUGUR_KV_EBOUNDS 2  /* an index addressed a slot/block/row outside its tensor */
#define AUGUR_KV_ECUDA 3    /* a CUDA runtime error; augur_kv_last_error() has the text */
#define AUGUR_KV_ETIMEOUT 4 /* a bounded device-side wait gave up */

/* Element types. Same-type copies are byte copies; mixed types convert through
 * fp32 with round-to-nearest-even, as torch's Tensor.copy_ does. */
#define AUGUR_KV_F32 0
#define AUGUR_KV_F16 1
#define AUGUR_KV_BF16 2

/* Flags for augur_kv_copy_runs. */
#define AUGUR_KV_COPY_AUTO 0   /* the measured-faster path for the layout (currently the vector path) */
#define AUGUR_KV_COPY_VECTOR 1 /* the 16/8/4/2/1-byte vector path */
#define AUGUR_KV_COPY_BULK 2   /* the TMA bulk path (EINVAL unless rows are dense and 16-byte aligned) */
/* OR-able: every thread ends with a system-scope fence, so the copy's stores
 * into another GPU's memory are performed before the kernel completes and a
 * ready flag written by later work on the stream cannot overtake them
 * (vector path; used for peer pushes). */
#define AUGUR_KV_COPY_FENCE_SYSTEM 4

/* Largest index passed by value to augur_kv_scatter (index_on_host = 1). */
#define AUGUR_KV_INLINE_INDEX_MAX 32

/* Library version, (major << 16) | minor. */
int augur_kv_version(void);

/* Text of the last error raised on this host thread ("" when none). */
const char* augur_kv_last_error(void);

/*
 * augur_kv_scatter — token scatter through a slot index: prefill K/V scatter
 * into the paged pool, the per-step decode append, and the contiguous-cache
 * write.
 *
 * Replaces the per-row index_put loop of write_kv (augur/kv_cache.py:103-106)
 * and the per-token loop of write_paged_kv (augur/paged_kv_cache.py:188-192);
 * with n_layers > 1 it is one launch for what the reference does in one call
 * per layer from attention (augur/attention.py:60,64-71).
 *
 * Source token t (0 <= t < n_tokens) of layer l, kv k (0 = K, 1 = V), head h:
 *   row = t / tokens_per_row, col = t % tokens_per_row
 *   src[k] + l*S[0] + row*S[1] + col*S[2] + h*S[3]     (S = src_k/v_strides)
 * Its destination slot:
 *   slot = row * index_row_base + index[row*index_strides[0] + col*index_strides[1]]
 *   dst[k] + l*D[0] + (slot / rows_per_major)*D[1] + (slot % rows_per_major)*D[2] + h*D[3]
 * A negative index skips the token (padding). index_row_base = 0 means the
 * index holds absolute slots (paged pool); index_row_base = rows_per_major
 * means it holds positions within row `row` (contiguous cache, row = batch).
 * An index >= rows_per_major with index_row_base > 0, or a slot >=
 * num_majors*rows_per_major, is an EBOUNDS error for that token.
 * index_on_host = 0: `index` is device memory read by the kernel.
 * index_on_host = 1: `index` is HOST memory; its n_tokens values (at most
 * AUGUR_KV_INLINE_INDEX_MAX, equal src/dst dtypes) are read during the call
 * and passed to the kernel by value, so a decode-step write needs no device
 * index buffer and no host-to-device copy.
 * head_dim elements are contiguous on both sides. src_v / dst_v may be NULL
 * (then only K moves). All strides are in elements of their own tensor.
 */
int augur_kv_scatter(const void* src_k, const void* src_v,
                     const int64_t* src_k_strides, /* [4] layer, row, col, head */
                     const int64_t* src_v_strides, /* [4] */
                     int64_t tokens_per_row, int32_t src_dtype,
                     void* dst_k, void* dst_v,
                     const int64_t* dst_strides, /* [4] layer, major, row, head */
                     int64_t rows_per_major, int64_t num_majors, int32_t dst_dtype,
                     const int64_t* index,         /* device, or host with index_on_host */
                     const int64_t* index_strides, /* [2] row, col */
                     int64_t index_row_base, int32_t index_on_host,
                     int64_t n_tokens, int32_t n_layers, int32_t n_heads, int32_t head_dim,
                     int32_t* status, /* device int32 or NULL */
                     void* stream);

/*
 * augur_kv_rope_scatter — rotary position embedding fused with the cache
 * write: rotates q (into q_out) and k by the table row of each token's
 * position, then writes the rotated k and the unchanged v to the cache. This
 * replaces apply_rope (augur/rope.py:12-40) followed by write_kv
 * (augur/kv_cache.py:75-112) or write_paged_kv (augur/paged_kv_cache.py:
 * 167-192), the sequence at augur/attention.py:53-71.
 *
 * Source addressing, the slot index and the destination follow
 * augur_kv_scatter (device index only; one dtype on every tensor). Token t
 * (row = t / tokens_per_row, col = t % tokens_per_row) has position
 * positions[row*position_strides[0] + col*position_strides[1]]. rope_cos and
 * rope_sin are [rope_positions][head_dim/2] tables in the cache dtype, built
 * like the reference's cos/sin (inv_freq = 1/theta^(2i/head_dim), angle =
 * position * inv_freq in float32, cos/sin cast to the dtype); element d and
 * d + head_dim/2 of a rotated row use entry d. q (n_q_heads heads, strides
 * [4] layer, row, col, head) is rotated into q_out (same shape); n_q_heads = 0
 * rotates k only. A token whose index is negative still has its q rotated.
 * Rounding matches the reference's three dtype ops (x*cos, rotate_half(x)*sin,
 * their sum), so the result is bit-exact given the same table. A position
 * outside [0, rope_positions) records AUGUR_KV_EBOUNDS and skips that token's
 * rotated rows.
 */
int augur_kv_rope_scatter(const void* src_k, const void* src_v,
                          const int64_t* src_k_strides, /* [4] layer, row, col, head */
                          const int64_t* src_v_strides, /* [4] */
                          int64_t tokens_per_row, int32_t dtype,
                          void* dst_k, void* dst_v,
                          const int64_t* dst_strides, /* [4] layer, major, row, head */
                          int64_t rows_per_major, int64_t num_majors,
                          const int64_t* index,         /* device */
                          const int64_t* index_strides, /* [2] row, col */
                          int64_t index_row_base,
                          const int64_t* positions,         /* device */
                          const int64_t* position_strides,  /* [2] row, col */
                          const void* rope_cos, const void* rope_sin, int64_t rope_positions,
                          const void* q, const int64_t* q_strides, /* [4] layer, row, col, head */
                          void* q_out, const int64_t* q_out_strides, int32_t n_q_heads,
                          int64_t n_tokens, int32_t n_layers, int32_t n_heads, int32_t head_dim,
                          int32_t* status, void* stream);

/*
 * augur_kv_copy_runs — copy runs of consecutive rows between two caches, all
 * layers, K and V, every head, in one launch. This is the block mover behind:
 *   - read_paged_kv, the logical-order gather (augur/paged_kv_cache.py:195-221)
 *   - copy_prefix_into_cache (augur/prefix_cache.py:53-75)
 *   - the contiguous->paged prefill handoff, which the reference expresses as
 *     write_paged_kv of cache.keys[l, b, :, :n_b] (augur/paged_kv_cache.py:167-192)
 *   - copy-on-write of a shared prefix block (no reference function; its
 *     result equals write_paged_kv of the copied rows into the new block).
 *
 * runs is a device int32 array [n_runs][5] = {src_major, src_row, dst_major,
 * dst_row, n_rows}. Run r, layer l, kv k, head h copies n_rows rows:
 *   src[k] + l*S[0] + src_major*S[1] + (src_row + i)*S[2] + h*S[3]
 *   -> dst[k] + l*D[0] + dst_major*D[1] + (dst_row + i)*D[2] + h*D[3]
 * for 0 <= i < n_rows. Rows must be dense (S[2] == D[2] == head_dim) for the
 * bulk path; other strides use the vector path. Bounds: src_major <
 * src_majors, src_row + n_rows <= src_rows_per_major, likewise for dst, and
 * n_rows <= max_rows; a run that fails them is skipped with EBOUNDS.
 * max_rows * head_dim * elem_size must be <= 16384 bytes.
 */
int augur_kv_copy_runs(const void* src_k, const void* src_v,
                       const int64_t* src_strides, /* [4] layer, major, row, head */
                       int64_t src_majors, int64_t src_rows_per_major, int32_t src_dtype,
                       void* dst_k, void* dst_v,
                       const int64_t* dst_strides, /* [4] */
                       int64_t dst_majors, int64_t dst_rows_per_major, int32_t dst_dtype,
                       const int32_t* runs, /* device [n_runs][5] */
                       int64_t n_runs, int32_t max_rows,
                       int32_t n_layers, int32_t n_heads, int32_t head_dim,
                       int32_t flags, int32_t* status, void* stream);

/*
 * augur_kv_paged_decode_attention — attention of one decode query per
 * sequence over its paged K/V, one layer, every sequence of the batch in one
 * launch. Replaces, for a decode step, read_paged_kv (the position-by-position
 * gather, augur/paged_kv_cache.py:195-221) plus the GQA repeat, the two
 * matmuls and the float32 softmax of augur/attention.py:72-86.
 *
 *   q       element (b, h, d) at q + b*q_strides[0] + h*q_strides[1] + d
 *           (n_q_heads rows per sequence, after RoPE)
 *   pools   one layer of the K and V pools: (block, kv_head, row, d) at
 *           pool + block*pool_strides[0] + kv_head*pool_strides[1]
 *           + row*pool_strides[2] + d
 *   tables  device int32 [batch][tables_stride]: logical block j of sequence
 *           b is block tables[b*tables_stride + j], j < max_blocks
 *   seq_lens device int32 [batch]; positions [0, seq_lens[b]) are attended;
 *           max_seq_len bounds them (host-known)
 *   out     element (b, h, d) at out + b*out_strides[0] + h*out_strides[1] + d
 * Query head h reads KV head h / (n_q_heads / n_kv_heads). The result equals
 * the reference's within floating-point tolerance (same rounding points,
 * different summation order). A block id outside [0, num_blocks) or a
 * position past max_blocks records AUGUR_KV_EBOUNDS and reads as zeros.
 * flags: AUGUR_KV_ATTN_AUTO picks the tensor-core kernel for bf16/fp16,
 * head_dim 64 or 128, <= 16 query heads per KV head; AUGUR_KV_ATTN_GENERIC
 * forces the CUDA-core kernel (any dtype; max_seq_len <= ~51,000).
 * counters / scratch: device memory for the split kernel, sized by
 * augur_kv_paged_decode_attention_workspace. counters (int32, 4-byte
 * aligned) must be zero before its first launch; every launch leaves it zero
 * and never stores data in it, so one counters buffer may serve launches of
 * any size one after another. scratch (16-byte aligned) needs no initial
 * contents. Launches that may run concurrently need their own counters and
 * scratch. With counters but too small a scratch (or none) every sequence is
 * processed unsplit; without counters, work items are also assigned statically.
 * A seq_lens entry above max_seq_len records AUGUR_KV_EBOUNDS and only its
 * first max_seq_len positions are attended. max_seq_len is at most 2^30.
 * flags | AUGUR_KV_ATTN_EARLY_READS (tensor-core kernel; ignored otherwise):
 * the launch is a programmatic dependent of the kernel ahead of it on the
 * stream either way; with this bit its CTAs read seq_lens, the block tables
 * and the K/V rows of their first work item BEFORE waiting for that kernel to
 * finish, so those reads overlap its last CTAs. Set it only when no work
 * still running at the launch writes seq_lens, the tables or this layer's
 * pool rows: the kernel ahead writes none of them, and everything before it
 * has finished (it has when the kernel ahead is a launch of this entry point
 * or of augur_kv_decode_layer, which release their dependents only after
 * their own wait). q, the new tokens' k / v (augur_kv_decode_layer), out and
 * the workspace are touched only after the wait, as without the bit.
 */
#define AUGUR_KV_ATTN_AUTO 0
#define AUGUR_KV_ATTN_GENERIC 1
#define AUGUR_KV_ATTN_EARLY_READS 16

int augur_kv_paged_decode_attention(const void* q, const int64_t* q_strides, /* [2] */
                                    const void* k_pool, const void* v_pool,
                                    const int64_t* pool_strides, /* [3] block, head, row */
                                    int64_t num_blocks, int32_t block_size,
                                    const int32_t* block_tables, int64_t tables_stride, int64_t max_blocks,
                                    const int32_t* seq_lens, int32_t max_seq_len, int32_t batch,
                                    int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype,
                                    void* out, const int64_t* out_strides, /* [2] */
                                    int32_t flags, int32_t* counters, int64_t counters_bytes,
                                    void* scratch, int64_t scratch_bytes, int32_t* status, void* stream);

/*
 * augur_kv_paged_prefill_attention — attention of a batch's new tokens (a
 * prefill, or the suffix of a prompt whose prefix blocks are already in the
 * pool) over the paged pool, one layer, reading every cached K/V row in place.
 * Replaces, for a whole batch, augur's paged branch after the write
 * (augur/attention.py:72-86: read_paged_kv, the GQA repeat, q k^T / sqrt(d),
 * the causal mask of _causal_mask (:15-19) with past_len = key_len -
 * query_len, the float32 softmax and P V), which the reference runs for a
 * batch of one (augur/paged_kv_cache.py:179-180).
 *
 *   q        query token j (after RoPE), head h: element d at
 *            q + j*q_strides[0] + h*q_strides[1] + d
 *   q_starts device int32 [batch + 1]: sequence b's query tokens are
 *            j in [q_starts[b], q_starts[b + 1]) (n_b of them, n_b <= max_q_len)
 *   seq_lens device int32 [batch]: cached positions of sequence b, its query
 *            tokens included (write them first); max_seq_len bounds them
 *   pool, block tables: as augur_kv_paged_decode_attention
 *   out      element (j, h, d) at out + j*out_strides[0] + h*out_strides[1] + d
 * Query token q_starts[b] + i sits at position seq_lens[b] - n_b + i and
 * attends to positions [0, seq_lens[b] - n_b + i]. Query head h reads KV head
 * h / (n_q_heads / n_kv_heads). The result equals the reference's within
 * floating-point tolerance (same rounding points, another summation order).
 * Lengths that disagree (n_b < 0, n_b > seq_lens[b], seq_lens[b] >
 * max_seq_len, n_b > max_q_len) record AUGUR_KV_EBOUNDS and skip that
 * sequence; a block id outside [0, num_blocks) records it and reads as zeros.
 * flags: AUGUR_KV_ATTN_AUTO takes the tcgen05 kernel (5th-generation tensor
 * cores, accumulators in tensor memory) for bf16/fp16, head_dim 64 or 128,
 * <= 8 query heads per KV head and 16-byte aligned rows of the pool, q and
 * out; the mma.sync kernel for the same shapes when q / out rows are only
 * 4-byte aligned; the CUDA-core kernel otherwise. AUGUR_KV_ATTN_TCGEN05 and
 * AUGUR_KV_ATTN_MMA_SYNC force those kernels (EINVAL for shapes they do not
 * take); AUGUR_KV_ATTN_GENERIC forces the CUDA-core kernel (any dtype;
 * max_seq_len <= ~51,000). Needs no workspace. A bounded wait of the tcgen05
 * kernel that gives up records AUGUR_KV_ETIMEOUT.
 */
#define AUGUR_KV_ATTN_TCGEN05 2
#define AUGUR_KV_ATTN_MMA_SYNC 3
int augur_kv_paged_prefill_attention(const void* q, const int64_t* q_strides, /* [2] token, head */
                                     const void* k_pool, const void* v_pool,
                                     const int64_t* pool_strides, /* [3] block, head, row */
                                     int64_t num_blocks, int32_t block_size,
                                     const int32_t* block_tables, int64_t tables_stride, int64_t max_blocks,
                                     const int32_t* seq_lens, const int32_t* q_starts, int32_t batch,
                                     int32_t max_q_len, int32_t max_seq_len, int32_t n_q_heads,
                                     int32_t n_kv_heads, int32_t head_dim, int32_t dtype,
                                     void* out, const int64_t* out_strides, /* [2] token, head */
                                     int32_t flags, int32_t* status, void* stream);

/*
 * augur_kv_paged_decode_attention_workspace — bytes of counters and scratch
 * that augur_kv_paged_decode_attention uses for these sizes on the current
 * device (0 and 0: none). No reference counterpart (the reference's eager
 * attention allocates its temporaries per call).
 */
int augur_kv_paged_decode_attention_workspace(int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                                              int32_t head_dim, int32_t max_seq_len, int32_t dtype,
                                              int32_t flags, int64_t* counters_bytes, int64_t* scratch_bytes);

/*
 * augur_kv_decode_layer — one layer of a batch's decode step, as one call:
 * the RoPE write of every sequence's new token (as augur_kv_rope_scatter) and
 * decode attention over each whole cached sequence (as
 * augur_kv_paged_decode_attention), on `stream`. For a decode step of
 * the whole batch this replaces augur's paged branch of attention
 * (augur/attention.py:53-86 with paged_cache: apply_rope, write_paged_kv,
 * read_paged_kv, the GQA repeat and the attention core), which the reference
 * runs for a batch of one (augur/paged_kv_cache.py:179-180,
 * augur/generation.py:35-40).
 *
 * args holds what every layer of the step shares and is filled once per step:
 * the pools, the step's slots and positions, the RoPE table, the block tables
 * and lengths (including the new token), the attention workspace and the
 * strides of q, key and value. Per layer: its index, the new token's q
 * (element (b, h, d) at q + b*q_strides[0] + h*q_strides[1] + d), key and
 * value (likewise with kv_strides) and out, a dense [batch][n_q_heads]
 * [head_dim] output.
 * The new token of sequence b is position seq_lens[b] - 1; positions[b] must
 * equal it and slots[b] must be its slot in the block table, as DecodeStep
 * and DecodeGraphStep build them. For bf16 / fp16 with head_dim 64 or 128
 * and <= 16 query heads per KV head (16-byte aligned rows), this is one
 * launch: the attention kernel rotates q and the new k itself and writes the
 * new k and v rows, bit for bit what the two separate launches write and
 * return. Other shapes run augur_kv_rope_scatter (the rotated q into
 * args->q_rot, otherwise unused scratch) and then the attention.
 * args->flags: as augur_kv_paged_decode_attention's. With
 * AUGUR_KV_ATTN_EARLY_READS the one-launch form reads the pool early (the
 * new token's row is loaded after the wait); the two-launch form drops the
 * bit, since its RoPE write just ahead writes the pool.
 * Returns the first failing code; AUGUR_KV_EINVAL for a null args or a layer
 * outside [0, n_layers).
 */
typedef struct augur_kv_decode_args {
  void* k_pool;                /* layer 0 of the K pool */
  void* v_pool;                /* layer 0 of the V pool (same strides) */
  int64_t pool_strides[4];     /* layer, block, kv_head, row (elements; head_dim contiguous) */
  int64_t num_blocks;
  int32_t block_size, n_layers, n_q_heads, n_kv_heads, head_dim, dtype, batch, flags;
  const int64_t* slots;        /* device [batch]: block * block_size + offset of each new token */
  const int64_t* positions;    /* device [batch]: position of each new token */
  const void* rope_cos;        /* device [rope_positions][head_dim / 2], cache dtype */
  const void* rope_sin;
  int64_t rope_positions;
  int64_t q_strides[2];        /* batch, head (elements) */
  int64_t kv_strides[2];       /* batch, head (elements) of key and value */
  void* q_rot;                 /* device [batch][n_q_heads][head_dim] */
  const int32_t* block_tables; /* device [batch][tables_stride] */
  int64_t tables_stride, max_blocks;
  const int32_t* seq_lens;     /* device [batch] */
  int32_t max_seq_len;
  int32_t launches;            /* out: kernels the latest augur_kv_decode_layer call launched (1 or 2) */
  int32_t* counters;           /* augur_kv_paged_decode_attention workspace */
  int64_t counters_bytes;
  void* scratch;
  int64_t scratch_bytes;
  int32_t* status;             /* device int32 or NULL */
} augur_kv_decode_args;

int augur_kv_decode_layer(augur_kv_decode_args* args, int32_t layer, const void* q, const void* key,
                          const void* value, void* out, void* stream);

/*
 * Peer memory for the disaggregated mode: a decode GPU's process exports its
 * block pool, a prefill GPU's process opens it and pushes finished blocks into
 * it with augur_kv_copy_runs (vector path: plain 16-byte stores over NVLink).
 * No reference counterpart (augur runs in one process on one device).
 *
 * augur_kv_ipc_export: handle (AUGUR_KV_IPC_HANDLE_BYTES bytes) of the device
 *   allocation containing dev_ptr, and dev_ptr's byte offset inside it.
 * augur_kv_ipc_open: map an exported allocation into the CURRENT device's
 *   address space (peer access is enabled as needed) and return the address
 *   that corresponds to `offset`. A process may not open its own allocation.
 * augur_kv_ipc_close: unmap what augur_kv_ipc_open returned (same offset).
 * The exporting process must keep the allocation alive until every importer
 * has closed it.
 */
#define AUGUR_KV_IPC_HANDLE_BYTES 64

int augur_kv_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int augur_kv_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out);
int augur_kv_ipc_close(void* dev_ptr, int64_t offset);

/*
 * Ready flags for the disaggregated handoff (no reference counterpart).
 * augur_kv_signal: a one-thread kernel on `stream` release-stores `value` to
 *   the int32 at `flag` (system scope; the flag may be another GPU's memory
 *   opened with augur_kv_ipc_open). Stream order puts it after the push.
 * augur_kv_wait: a one-thread kernel on `stream` that spins with acquire
 *   loads until *flag >= value, for at most timeout_ns (0 < timeout_ns <=
 *   60 s) of %globaltimer time; on timeout it writes AUGUR_KV_ETIMEOUT to the
 *   status word and returns, so later work on the stream runs and the
 *   context stays usable. Work queued after the wait on the same stream is
 *   ordered after the flag (or the timeout).
 * A signaller and its waiter must run on different GPUs: two launches on one
 * GPU are not guaranteed to run at the same time.
 */
int augur_kv_signal(int32_t* flag, int32_t value, void* stream);
int augur_kv_wait(const int32_t* flag, int32_t value, int64_t timeout_ns, int32_t* status, void* stream);

/*
 * augur_kv_copy_runs_noalloc — augur_kv_copy_runs for callers that cannot
 * allocate device memory. No counterpart in the reference (augur allocates
 * through torch).
 *
 * augur_kv_copy_runs reads its run list from a device buffer the caller must
 * allocate. Some callers cannot call cudaMalloc: an engine whose device memory
 * is one up-front reservation carved into cache blocks by its own allocator
 * (an extra allocation would fail or break its accounting), or a plain C/C++
 * host without a device allocator of its own. This variant takes the run list
 * in HOST memory (same [n_runs][5] layout) and stages it in a fixed array
 * inside the library (a file-scope __device__ array of
 * AUGUR_KV_NOALLOC_MAX_RUNS runs, 1.25 MiB, held by every GPU that loads the
 * library until the process exits); the caller still passes the caches
 * themselves. It calls no cudaMalloc, cudaFree or other allocating routine.
 *
 * - n_runs > AUGUR_KV_NOALLOC_MAX_RUNS is rejected with AUGUR_KV_EINVAL.
 * - The first call on each device with work to do (n_runs > 0; a call with
 *   no runs returns before this) looks up the array's device address
 *   (cudaGetSymbolAddress). Under lazy module loading (the CUDA 12 default)
 *   that lookup may load this library's module onto the device and commit
 *   the array there, so make that first call before the engine reserves its
 *   device memory and before any stream capture.
 * - Every argument check runs before anything is staged: a call rejected
 *   with AUGUR_KV_EINVAL leaves the array as it was.
 * - host_runs is read by a stream-ordered host-to-device copy: pageable memory
 *   may be reused when the call returns; pinned memory must stay unchanged
 *   until the stream has passed this call.
 * - Every call shares the one array. Calls whose work overlaps on the GPU
 *   (issued on different streams without ordering) race on it.
 * Everything else (arguments, bounds checks, status word) is as for
 * augur_kv_copy_runs.
 */
#define AUGUR_KV_NOALLOC_MAX_RUNS 65536

int augur_kv_copy_runs_noalloc(const void* src_k, const void* src_v,
                               const int64_t* src_strides, /* [4] */
                               int64_t src_majors, int64_t src_rows_per_major, int32_t src_dtype,
                               void* dst_k, void* dst_v,
                               const int64_t* dst_strides, /* [4] */
                               int64_t dst_majors, int64_t dst_rows_per_major, int32_t dst_dtype,
                               const int32_t* host_runs, /* HOST [n_runs][5] */
                               int64_t n_runs, int32_t max_rows,
                               int32_t n_layers, int32_t n_heads, int32_t head_dim,
                               int32_t flags, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AUGUR_KV_H */
