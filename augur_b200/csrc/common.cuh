// common.cuh — helpers shared by the source files of libaugur_kv.so (internal).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace augur_kv_dev {

constexpr int kMaxDevices = 64;

// Text of the last error on this host thread (augur_kv_last_error).
extern thread_local char g_last_error[512];
// Guards the per-device launch-configuration caches (recursive: cached
// queries such as sm_count may run while a caller holds it).
extern std::recursive_mutex g_cache_mutex;

// Record an error message and return `code`.
int fail(int code, const char* fmt, ...);
// AUGUR_KV_ECUDA with the runtime's message if the last launch failed.
int check_launch(const char* what);
// Bytes per element of an AUGUR_KV_* dtype (0 if unknown).
int elem_size(int32_t dtype);
// SM count of the current device (cached).
int sm_count();
// Resident CTAs per SM of `kernel` at `threads` threads, no dynamic shared
// memory (occupancy calculator; cached per device and kernel).
int resident_ctas(const void* kernel, int threads);

// The RoPE write of a decode step's new tokens, fused into the decode
// attention launch: new k / v (element (b, h, d) at + b*new_stride_b +
// h*new_stride_h + d, element strides), the cos / sin tables and their rows.
struct FusedRope {
  const void* new_k;
  const void* new_v;
  int64_t new_stride_b, new_stride_h;
  const void* cos;
  const void* sin;
  int64_t n_pos;
  // the step's positions and slots as the caller built them (device int64
  // [batch], or both null): checked against seq_lens - 1 and the block table
  const int64_t* positions;
  const int64_t* slots;
};

// augur_kv_paged_decode_attention, optionally with `fuse`: q is then before
// RoPE, position seq_lens[b] - 1 of each sequence is its new token, taken
// from fuse->new_k / new_v, rotated, attended and written to its pool row.
// With `fuse`, *fused says whether the fused launch was issued; when it was
// not (the shape or alignment needs the generic kernel), nothing was
// launched and the call returned AUGUR_KV_OK.
int paged_decode_attention_impl(const void* q, const int64_t* q_strides, const void* k_pool, const void* v_pool,
                                const int64_t* pool_strides, int64_t num_blocks, int32_t block_size,
                                const int32_t* block_tables, int64_t tables_stride, int64_t max_blocks,
                                const int32_t* seq_lens, int32_t max_seq_len, int32_t batch, int32_t n_q_heads,
                                int32_t n_kv_heads, int32_t head_dim, int32_t dtype, void* out,
                                const int64_t* out_strides, int32_t flags, int32_t* counters, int64_t counters_bytes,
                                void* scratch, int64_t scratch_bytes, int32_t* status, void* stream,
                                const FusedRope* fuse, bool* fused);

// First device-side error wins.
__device__ __forceinline__ void record_status(int32_t* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// RoPE of two packed element pairs (x1 from the first half of a row, x2 the
// same dims of the second half) with packed cos / sin c, s, in the cache
// dtype: x1' = x1 c - x2 s, x2' = x2 c + x1 s, each product and the sum
// rounded to the dtype as the reference's three tensor ops round them (the
// single definition rope_scatter_kernel and the fused decode attention both
// use, so the fused and separate RoPE writes give the same bits). Each
// packed op rounds the exact result once; the reference rounds the float32
// result (itself exact for the products) to T, and since 24 >= 2 x 11 + 2
// that double rounding gives the same bits. The explicit .rn keeps the
// compiler from contracting a product and a sum into a fused multiply-add.
template <typename T>
__device__ __forceinline__ void rope_pair(uint32_t& x1, uint32_t& x2, uint32_t c, uint32_t s);
#define AUGUR_KV_ROPE_PAIR(TYPE, SUFFIX)                                                         \
  template <>                                                                                      \
  __device__ __forceinline__ void rope_pair<TYPE>(uint32_t & x1, uint32_t & x2, uint32_t c, uint32_t s) { \
    uint32_t ac, bs, bc, as;                                                                        \
    asm("mul.rn." SUFFIX " %0, %1, %2;" : "=r"(ac) : "r"(x1), "r"(c));                              \
    asm("mul.rn." SUFFIX " %0, %1, %2;" : "=r"(bs) : "r"(x2), "r"(s));                              \
    asm("mul.rn." SUFFIX " %0, %1, %2;" : "=r"(bc) : "r"(x2), "r"(c));                              \
    asm("mul.rn." SUFFIX " %0, %1, %2;" : "=r"(as) : "r"(x1), "r"(s));                              \
    asm("sub.rn." SUFFIX " %0, %1, %2;" : "=r"(x1) : "r"(ac), "r"(bs));                             \
    asm("add.rn." SUFFIX " %0, %1, %2;" : "=r"(x2) : "r"(bc), "r"(as));                             \
  }
AUGUR_KV_ROPE_PAIR(__nv_bfloat16, "bf16x2")
AUGUR_KV_ROPE_PAIR(__half, "f16x2")
#undef AUGUR_KV_ROPE_PAIR

}  // namespace augur_kv_dev
