// augur_attn.cu — decode attention that reads the paged KV pool directly.
//
// The reference computes a decode step's attention by gathering the whole
// sequence out of the pool position by position (read_paged_kv,
// augur/paged_kv_cache.py:217-220), repeating each K/V head for the query
// heads of its group and running two eager matmuls around a float32
// softmax (augur/attention.py:72-86). Here one launch covers every sequence
// of the batch for one layer, reading each K/V row of the pool once:
//
//  * attn_decode_split_kernel (bf16 / fp16, head_dim 64 or 128, <= 16 query
//    heads per KV head): a persistent grid of the resident CTAs. Sequences
//    are cut into chunks of equal size (a power-of-two multiple of warps x 32
//    tokens) that each CTA derives on the device from seq_lens so the work
//    items, (sequence, KV head, chunk) triples numbered in order, number at
//    most four waves of the grid; CTA i takes item i, then items from an
//    atomic counter. Each warp stages 32 tokens of K and V in shared memory
//    with cp.async and runs both products transposed on mma.sync m16n8k16
//    (tokens, not the few query heads of a group, fill the 16 rows) around
//    an online softmax. Chunks of one sequence combine through
//    caller-provided counters and scratch: the last CTA to arrive (an atomic
//    counter; no CTA ever waits) merges the partials and writes the output.
//    Its fused instance (template argument FUSE, launched only for
//    augur_kv_decode_layer) also does the decode step's RoPE write, which
//    the reference runs first (apply_rope then write_paged_kv,
//    augur/attention.py:53-71):
//      - q arrives before RoPE and is rotated in registers;
//      - the new token (position seq_len - 1) is staged from the layer's k
//        and v inputs instead of the pool, its k rotated in shared memory;
//      - the owning warp writes that k and v to the token's pool row.
//    The rotation uses the same packed ops as rope_scatter_kernel, so the
//    results are those of the two separate launches, bit for bit.
//  * attn_decode_generic_kernel (any dtype / shape): one CTA per (sequence,
//    query head), scores of the whole sequence in shared memory, then the
//    reference's order of operations: max, exp, sum, normalise, P.V.
//
// Rounding follows the reference where it rounds: scores are rounded to the
// cache dtype after q.k and again after the division by sqrt(head_dim)
// (the bf16/fp16 matmul output and the scalar division both produce the
// dtype; for bf16 with sqrt(head_dim) a power of two the division is an
// exact scaling of a bf16 value, so the second rounding changes nothing and
// the split kernel skips it); probabilities are rounded before the product
// with V; the output is rounded once. The split kernel evaluates exp as
// 2^(x log2 e) with the ex2.approx instruction (relative error about 2^-22,
// far below the bf16/fp16 rounding that follows). Summation order differs,
// so results agree within a floating-point tolerance, not bit for bit.
//
// The decode query sits at the last position of its sequence, so the causal
// mask hides nothing; tokens at or past seq_len are never read.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

#include "augur_kv.h"
#include "common.cuh"

namespace augur_kv_dev {

struct AttnArgs {
  const char* q;
  int64_t q_stride_b, q_stride_h;  // bytes
  const char* k;
  const char* v;
  int64_t blk_stride, head_stride, row_stride;  // bytes; head_dim contiguous
  int64_t num_blocks;
  int32_t block_size;
  const int32_t* tables;
  int64_t tables_stride;  // elements
  int64_t max_blocks;     // columns of the block table
  const int32_t* seq_lens;
  int32_t batch, hq, hkv, groups, head_dim;
  float sqrt_d;
  float inv_sqrt_d;     // 1 / sqrt_d, used when multiplying by it equals dividing
  int32_t scale_exact;  // sqrt_d is a power of two
  char* out;
  int64_t out_stride_b, out_stride_h;  // bytes
  int32_t dtype;
  int32_t max_seq;   // max_seq_len: bound on seq_lens (generic kernel: score capacity)
  int32_t bs_shift;  // log2(block_size) when it is a power of two, else -1
  // split kernel
  int32_t chunk;      // smallest chunk size the plan may pick (a power of two)
  int32_t max_items;  // work items the plan may create (waves x grid); partial slots in the scratch
  int32_t* ws_sched;  // counters [0]: next item to hand out, [1]: CTAs done (null: static items)
  int32_t* ws_cnt;
  float* ws_ml;
  float* ws_o;
  int32_t* status;
  // RoPE write of a decode step's new tokens fused into the attention launch
  // (augur_kv_decode_layer): q is before RoPE, and position seq_len - 1 of
  // each sequence is its new token, whose k and v come from new_k / new_v
  // (element (b, h, d) at + b*new_stride_b + h*new_stride_h + d*2); the
  // rotated k and the v are written to that position's pool row here.
  int32_t fuse;
  const char* new_k;
  const char* new_v;
  int64_t new_stride_b, new_stride_h;  // bytes
  const char* rope_cos;  // [rope_n][head_dim / 2] in the cache dtype
  const char* rope_sin;
  int64_t rope_n;
  char* k_w;  // the pools, writable (fused launches only)
  char* v_w;
  // fused launches: the step's positions and slots as the caller built them
  // (may be null). The kernel takes the new token's position from seq_len - 1
  // and its slot from the block table; it records AUGUR_KV_EBOUNDS where
  // these disagree with them (the two-launch path uses them directly).
  const int64_t* chk_pos;
  const int64_t* chk_slot;
  // AUGUR_KV_ATTN_EARLY_READS: seq_lens, the block tables and the pool rows
  // of a CTA's first item are read before the grid-dependency wait
  int32_t early;
};

constexpr float kNegInf = -INFINITY;

__device__ __forceinline__ int elem_size_dev(int dtype) { return dtype == AUGUR_KV_F32 ? 4 : 2; }

__device__ __forceinline__ float load_elem(const char* p, int dtype) {
  if (dtype == AUGUR_KV_F32) return *reinterpret_cast<const float*>(p);
  if (dtype == AUGUR_KV_F16) return __half2float(*reinterpret_cast<const __half*>(p));
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
}

// Value after rounding to the cache dtype (what a tensor of that dtype holds).
__device__ __forceinline__ float round_to(float x, int dtype) {
  if (dtype == AUGUR_KV_F16) return __half2float(__float2half_rn(x));
  if (dtype == AUGUR_KV_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  return x;
}

__device__ __forceinline__ void store_elem(char* p, int dtype, float x) {
  if (dtype == AUGUR_KV_F32) *reinterpret_cast<float*>(p) = x;
  else if (dtype == AUGUR_KV_F16) *reinterpret_cast<__half*>(p) = __float2half_rn(x);
  else *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16_rn(x);
}

// Address of K or V row `pos` of sequence b, KV head hk; nullptr (and EBOUNDS)
// for a block id outside the pool.
__device__ __forceinline__ const char* row_addr(const AttnArgs& a, const char* pool, int b, int hk, int pos) {
  const int lb = pos / a.block_size;
  if (lb >= a.max_blocks) {
    record_status(a.status, AUGUR_KV_EBOUNDS);
    return nullptr;
  }
  const int blk = __ldg(a.tables + int64_t(b) * a.tables_stride + lb);
  if (blk < 0 || blk >= a.num_blocks) {
    record_status(a.status, AUGUR_KV_EBOUNDS);
    return nullptr;
  }
  return pool + int64_t(blk) * a.blk_stride + int64_t(hk) * a.head_stride +
         int64_t(pos - lb * a.block_size) * a.row_stride;
}

// ---------------------------------------------------------------------------
// Tensor-core path
// ---------------------------------------------------------------------------

template <typename T> struct MmaType;
template <> struct MmaType<__nv_bfloat16> {
  static constexpr int dtype = AUGUR_KV_BF16;
};
template <> struct MmaType<__half> {
  static constexpr int dtype = AUGUR_KV_F16;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 8-byte async copy global -> shared (both addresses 8-byte aligned).
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// 16-byte async copy global -> shared; src_bytes = 0 writes 16 zero bytes.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

constexpr int kStageTok = 32;       // tokens a warp stages and processes at a time
constexpr int kMaxChunks = 256;     // chunks per (sequence, KV head)
constexpr int kMaxSeq = 1 << 30;    // longest sequence a launch accepts

// Launch shape of the split kernel for one head_dim and NS stage buffers per
// warp: each buffer holds 32 tokens of K and V rows, padded so ldmatrix rows
// hit distinct banks. The shared memory stays the same for NS = 1 and 2 (half
// the warps, each with two buffers, so a warp prefetches its next stage).
// Chunks are multiples of warps x 32 tokens.
template <int D, int NS>
struct SplitCfg {
  static constexpr int kWarps = (D == 64 ? 8 : 4) / NS;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kChunkUnit = kWarps * kStageTok;
  static constexpr int kRowBytes = D * 2 + 16;
  static constexpr int kStageBytes = kStageTok * kRowBytes;  // K or V of one stage
  static constexpr int kWarpStage = 2 * kStageBytes;
  static constexpr int kPipe = kWarps * NS * kWarpStage;
  // after the token loop the warps' partial results reuse the stage buffers
  static constexpr int kPO = D + 4;  // floats per partial row: the transposing stores hit distinct banks
  static_assert((16 * kPO + 32) * 4 <= NS * kWarpStage, "a warp's partial must fit in its stage buffers");
  static_assert(2 * kMaxChunks * 16 * 4 <= kPipe, "chunk maxima and sums must fit in the stage buffers");
  // fac, cta_m, cta_l, flag, 2 item descriptors; then, for fused launches,
  // the new token's cos and sin rows and its pool offset
  static constexpr int kTailNew = 768;
  static_assert((kWarps * 16 + 16 + 16 + 16) * 4 + 2 * 6 * 4 <= kTailNew, "tail layout");
  // pool offset, then the caller's position and slot of the new token, as read
  static constexpr int kTail = kTailNew + D * 2 + 32;
  static constexpr int kBytes = kPipe + kTail;
};

#ifndef AUGUR_KV_ATTN_STAGES
#define AUGUR_KV_ATTN_STAGES 1  // stage buffers per warp at head_dim 64
#endif
#ifndef AUGUR_KV_ATTN_COMBINE_REGS
#define AUGUR_KV_ATTN_COMBINE_REGS 20  // registers per thread holding partial outputs in the combine
#endif

__device__ __forceinline__ float ex2(float x) {  // 2^x; ex2(-inf) = 0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// atomicAdd with acquire-release semantics at GPU scope; returns the old value.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Transpose an 8x8 matrix of 16-bit values held as the mma fragment layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Round two floats to the cache dtype and back (what a tensor of that dtype holds).
template <typename T>
__device__ __forceinline__ float2 round2(float x, float y);
template <>
__device__ __forceinline__ float2 round2<__nv_bfloat16>(float x, float y) {
  return __bfloat1622float2(__floats2bfloat162_rn(x, y));
}
template <>
__device__ __forceinline__ float2 round2<__half>(float x, float y) {
  return __half22float2(__floats2half2_rn(x, y));
}

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// C is a power of two (a power-of-two chunk unit times 2^j)
__device__ __forceinline__ int chunks_of(int S, int C) { return max(1, (S + C - 1) >> (__ffs(C) - 1)); }

// Work items are (sequence, KV head, chunk) triples numbered sequence-major,
// then KV head, then chunk, so the chunks of one (sequence, KV head) are
// consecutive. Every CTA's warp 0 derives the same plan from seq_lens: the
// smallest chunk size C = a.chunk * 2^j for which the items number at most
// a.max_items (a few waves of the persistent grid, so the longest sequence is
// spread over several CTAs), or C >= max_seq_len (one chunk per sequence; also
// when the (sequence, KV head) units alone exceed a.max_items).
struct Plan {
  int C, total;
};

__device__ __forceinline__ int seq_len_at(const AttnArgs& a, int b) {
  return min(max(0, __ldg(a.seq_lens + b)), a.max_seq);
}

// Batches up to kResidentSeqs keep each sequence's item count in warp 0's
// registers (lane l holds sequences l, l + 32, l + 64, l + 96), so finding an
// item needs no memory access.
constexpr int kResidentSeqs = 128;

__device__ Plan make_plan(const AttnArgs& a, int lane, int (&rc)[4]) {
  Plan p;
  p.C = a.chunk;
  const int64_t units = int64_t(a.batch) * a.hkv;
  if (units > int64_t(a.max_items) || p.C >= a.max_seq) {  // one chunk per sequence
    p.C = max(p.C, a.max_seq);
    p.total = int(units);
    return p;
  }
  // the first 256 lengths in registers, loaded in one round; the rest (larger
  // batches) re-read per candidate, four loads in flight at a time
  constexpr int kRegSeqs = 8;
  int sl[kRegSeqs];
#pragma unroll
  for (int k = 0; k < kRegSeqs; ++k) {
    const int b = lane + 32 * k;
    sl[k] = b < a.batch ? seq_len_at(a, b) : -1;
  }
  for (;;) {
    int cnt = 0;
#pragma unroll
    for (int k = 0; k < kRegSeqs; ++k) cnt += sl[k] >= 0 ? chunks_of(sl[k], p.C) : 0;
#pragma unroll 4
    for (int b = lane + 32 * kRegSeqs; b < a.batch; b += 32) cnt += chunks_of(seq_len_at(a, b), p.C);
    p.total = warp_sum(cnt) * a.hkv;
    if (p.total <= a.max_items || p.C >= a.max_seq) break;
    p.C *= 2;
  }
  if (a.batch <= kResidentSeqs) {
#pragma unroll
    for (int k = 0; k < 4; ++k) rc[k] = sl[k] >= 0 ? chunks_of(sl[k], p.C) * a.hkv : 0;
  }
  return p;
}

struct Item {
  int b, hk, chunk, nch, first;  // first: item number of chunk 0 of (b, hk)
};

// Position of warp 0's search over seq_lens: the items of sequences < b number base.
struct Cursor {
  int b, base;
};

// Item `item` of the plan. A CTA visits its items in increasing order, so the
// search resumes from the cursor (sequences before it hold only earlier items).
__device__ Item locate(const AttnArgs& a, const Plan& p, int item, int lane, const int (&rc)[4], Cursor& cur) {
  Item it;
  if (p.C >= a.max_seq) {  // every sequence is one chunk
    it.b = item / a.hkv;
    it.hk = item - it.b * a.hkv;
    it.chunk = 0;
    it.nch = 1;
    it.first = item;
    return it;
  }
  // cursor: resident batches scan from group cur.b / 32 of the register counts;
  // others re-read seq_lens from sequence cur.b on
  const bool resident = a.batch <= kResidentSeqs;
  for (;;) {
    const int b = cur.b + lane;
    int c;
    if (resident) {
      const int k = cur.b >> 5;
      c = k == 0 ? rc[0] : k == 1 ? rc[1] : k == 2 ? rc[2] : rc[3];
    } else {
      c = b < a.batch ? chunks_of(seq_len_at(a, b), p.C) * a.hkv : 0;
    }
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, c > 0 && item >= cur.base + incl - c && item < cur.base + incl);
    if (hit != 0u) {
      const int src = __ffs(hit) - 1;
      const int base = cur.base + __shfl_sync(0xffffffffu, incl - c, src);
      it.nch = __shfl_sync(0xffffffffu, c, src) / a.hkv;
      it.b = cur.b + src;
      const int rel = item - base;
      it.hk = rel / it.nch;
      it.chunk = rel - it.hk * it.nch;
      it.first = base + it.hk * it.nch;
      if (!resident) {  // resident: the cursor stays at the start of this group of 32
        cur.b = it.b;
        cur.base = base;
      }
      return it;
    }
    cur.base += __shfl_sync(0xffffffffu, incl, 31);
    cur.b += 32;
  }
}

// Each work item is a chunk of C tokens of one (sequence, KV head), and a CTA
// processes its items one after another. Each warp takes every kWarps-th
// 32-token stage of the chunk (NS stage buffers per warp) and stages its
// K and V rows in shared memory with cp.async (one block-table entry per lane
// per stage, shared by shuffle). Both products run transposed on mma.sync
// m16n8k16 so the stage's tokens, not the few query heads of the group, fill
// the 16 rows: S^T = K Q^T (16 tokens x 8 heads per tile), then, after an
// online softmax in base 2 on the columns, O^T += V^T P^T (16 dims x 8 heads)
// with P^T moved into the B-operand layout by movmatrix. NT = 1 serves up to
// 8 query heads per KV head, NT = 2 up to 16. Warps combine in shared memory.
// A sequence of one chunk writes its output directly; otherwise each CTA
// writes its unnormalised partial (o, m, l) to the scratch slot of its item
// and the last CTA of the (sequence, KV head) to arrive (atomic counter, no
// waiting) combines them and resets the counter.
template <typename T, int D, int NT, int NS, bool FUSE>
__global__ void __launch_bounds__(SplitCfg<D, NS>::kThreads, (D == 64 && NT == 1) ? 3 * NS : 1)
    attn_decode_split_kernel(AttnArgs a) {
  using CF = SplitCfg<D, NS>;
  constexpr int W = CF::kWarps;
  constexpr int DT = MmaType<T>::dtype;
  constexpr int PARTS = D * 2 / 16;         // 16-byte pieces per row
  constexpr int ROW_STEP = 32 / PARTS;      // row distance between a lane's rows
  constexpr int RPL = kStageTok / ROW_STEP; // rows per lane per stage
  constexpr int PO = CF::kPO;
  extern __shared__ __align__(128) unsigned char smem[];
  // after the token loop warp w's partial sits in its own stage buffers:
  // wwpart[w * WSF + head * PO + dim], maxima at + 16 PO, sums at + 16 PO + 16
  const float* wpart = reinterpret_cast<const float*>(smem);
  constexpr int WSF = NS * CF::kWarpStage / 4;
  float* fac = reinterpret_cast<float*>(smem + CF::kPipe);  // [warps][16]
  float* cta_m = fac + W * 16;
  float* cta_l = cta_m + 16;
  int* last_flag = reinterpret_cast<int*>(cta_l + 16);
  // fused launches: the new token's cos and sin rows, then its pool offset
  unsigned char* new_cs = smem + CF::kPipe + CF::kTailNew;
  unsigned char* new_sn = new_cs + D;
  int64_t* new_ofs = reinterpret_cast<int64_t*>(new_sn + D);
  int64_t* new_chk = new_ofs + 1;  // [0] caller's position, [1] caller's slot, [2] the table's slot

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  // Launched as a programmatic dependent of the previous kernel on the
  // stream: wait for it to finish (its writes visible) before reading inputs.
  // With early reads the plan, the first item's block-table entries and its
  // K/V rows are read first, while the previous kernel's last CTAs drain; q,
  // the new token's k / v, the output and the workspace only after the wait.
  const bool early = a.early != 0;
  if (!early) asm volatile("griddepcontrol.wait;" ::: "memory");
  // Persistent: CTA i takes items i, i + grid, i + 2 grid, ... Warp 0 plans,
  // then finds each item one item ahead (while its own loads for the current
  // item are in flight) and publishes it in a double-buffered descriptor.
  int* desc = last_flag + 1;  // [2][6]: C, b, hk, chunk, nch, first (b = -1: no item)
  Plan plan{0, 0};
  Cursor cur{0, 0};
  int rc[4] = {0, 0, 0, 0};  // warp 0: item counts of sequences lane + 32 k (batches <= 128)
  auto publish = [&](int slot, int id) {  // warp 0, all lanes
    int* d = desc + slot * 6;
    if (id < plan.total) {
      const Item itm = locate(a, plan, id, lane, rc, cur);
      if (lane == 0) {
        d[0] = plan.C;
        d[1] = itm.b;
        d[2] = itm.hk;
        d[3] = itm.chunk;
        d[4] = itm.nch;
        d[5] = itm.first;
      }
    } else if (lane == 0) {
      d[1] = -1;
    }
  };
  // CTA i's first item is i; later ones come from an atomic counter (items
  // grid, grid + 1, ...) when there are counters, the last CTA to finish
  // resetting it, else CTA i takes i + grid, i + 2 grid, ...
  int32_t* sched = a.ws_sched;
  int static_next = blockIdx.x;
  auto next_id = [&]() -> int {  // warp 0, all lanes
    int id = static_next;
    if (sched != nullptr && static_next >= int(gridDim.x)) {
      if (lane == 0) id = int(gridDim.x) + atomicAdd(sched, 1);
      id = __shfl_sync(0xffffffffu, id, 0);
    }
    static_next += gridDim.x;
    return id;
  };
  if (warp == 0) {
    plan = make_plan(a, lane, rc);
    publish(0, next_id());
  }
  bool first_item = true;
  int slot = 0;
  for (;; slot ^= 1) {
  __syncthreads();  // descriptor `slot` is published; the previous item is done with shared memory
  const int* d = desc + slot * 6;
  if (d[1] < 0) {
    if (early && first_item) asm volatile("griddepcontrol.wait;" ::: "memory");  // before the workspace
    if (sched != nullptr && threadIdx.x == 0 && atomicAdd(sched + 1, 1) == int(gridDim.x) - 1) {
      sched[0] = 0;  // every CTA has taken its last id: ready for the next launch
      sched[1] = 0;
    }
    return;
  }
  const int plan_C = d[0], b = d[1], hk = d[2], chunk = d[3];
  const int my_nch = d[4], item_first = d[5];
  const int S = seq_len_at(a, b);
  if (chunk == 0 && threadIdx.x == 0 && __ldg(a.seq_lens + b) > a.max_seq)
    record_status(a.status, AUGUR_KV_EBOUNDS);  // the host sized the launch with max_seq_len
  const int tok0 = chunk * plan_C, tok1 = min(S, tok0 + plan_C);
  const int G = a.groups;

  // Q^T as mma B fragments (loaded once this item's first K/V loads are issued)
  uint32_t qb[D / 16][NT][2];
  // O^T accumulators: o[dm][nt] = O^T[dims dm*16 + g (+8)][heads nt*8 + 2t (+1)]
  float o[D / 16][NT][4];
#pragma unroll
  for (int i = 0; i < D / 16; ++i)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[i][nt][0] = o[i][nt][1] = o[i][nt][2] = o[i][nt][3] = 0.f;
  // base-2 running max and lane-partial sums of the lane's two head columns per n-tile
  float mrow[NT][2], lrow[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) mrow[nt][0] = mrow[nt][1] = kNegInf, lrow[nt][0] = lrow[nt][1] = 0.f;

  unsigned char* wbuf = smem + warp * NS * CF::kWarpStage;
  const int part = lane % PARTS, row0 = lane / PARTS;
  const int new_pos = FUSE ? S - 1 : -1;  // fused launches: the step's new token
  const int64_t lane_off = int64_t(hk) * a.head_stride + part * 16;
  const int32_t* tbl = a.tables + int64_t(b) * a.tables_stride;
  const int shift = a.bs_shift;
  // Stage tokens [s0, s0 + 32) into buffer buf: lane l reads the table entry
  // of the stage's l-th logical block (a stage spans at most 32 blocks).
  // the new token's cos / sin rows to the tail and (lane part 0) the caller's
  // position and slot, compared when the row is written
  auto load_new_inputs = [&](int pos) {
    if (part == 0 && a.chk_pos != nullptr) {
      cp_async8(new_chk, a.chk_pos + b);
      cp_async8(new_chk + 1, a.chk_slot + b);
    }
    if (part < PARTS / 2) {
      const bool in_table = pos < a.rope_n;
      const int64_t row = in_table ? int64_t(pos) * D : 0;  // D/2 elements of 2 bytes
      cp_async16(new_cs + part * 16, a.rope_cos + row + part * 16, in_table ? 16 : 0);
      cp_async16(new_sn + part * 16, a.rope_sin + row + part * 16, in_table ? 16 : 0);
      if (!in_table && part == 0) record_status(a.status, AUGUR_KV_EBOUNDS);
    }
  };
  // late: the new token's row of a fused launch is left to load_new_late
  // (after the grid-dependency wait); its pool offset is still recorded here
  auto load_stage = [&](int s0, int buf, bool late) {
    const int last = min(tok1, s0 + kStageTok) - 1;
    const int lb_first = shift >= 0 ? (s0 >> shift) : s0 / a.block_size;
    const int lb_last = shift >= 0 ? (last >> shift) : last / a.block_size;
    int my_blk = -1;
    if (lb_first + lane <= lb_last && lb_first + lane < a.max_blocks) my_blk = __ldg(tbl + lb_first + lane);
    unsigned char* kdst = wbuf + buf * CF::kWarpStage + part * 16;
    unsigned char* vdst = kdst + CF::kStageBytes;
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      const int r = row0 + i * ROW_STEP;
      const int pos = s0 + r;
      int lb, off;
      if (shift >= 0) {
        lb = pos >> shift;
        off = pos & (a.block_size - 1);
      } else {
        lb = pos / a.block_size;
        off = pos - lb * a.block_size;
      }
      const int blk = __shfl_sync(0xffffffffu, my_blk, (lb - lb_first) & 31);
      const char* kp = a.k;
      const char* vp = a.v;
      int bytes = 0;
      if (pos < tok1) {
        const bool blk_ok = blk >= 0 && blk < a.num_blocks;
        if (blk_ok) {
          const int64_t ofs = int64_t(blk) * a.blk_stride + lane_off + int64_t(off) * a.row_stride;
          kp += ofs;
          vp += ofs;
          bytes = 16;
        } else {
          record_status(a.status, AUGUR_KV_EBOUNDS);  // reads as zeros
        }
        if (FUSE && pos == new_pos) {  // the new token: its k and v from the inputs, its cos / sin rows to the tail
          if (part == 0) {
            *new_ofs = blk_ok ? int64_t(blk) * a.blk_stride + int64_t(hk) * a.head_stride +
                                    int64_t(off) * a.row_stride
                              : int64_t(-1);
            new_chk[2] = int64_t(blk) * a.block_size + off;
          }
          if (late) continue;
          load_new_inputs(pos);
          const int64_t src = int64_t(b) * a.new_stride_b + int64_t(hk) * a.new_stride_h + part * 16;
          kp = a.new_k + src;
          vp = a.new_v + src;
          bytes = 16;
        }
      }
      cp_async16(kdst + r * CF::kRowBytes, kp, bytes);
      cp_async16(vdst + r * CF::kRowBytes, vp, bytes);
    }
    cp_async_commit();
  };
  // the new token's row of stage s0 (a fused launch's first stage loaded
  // with late = true): its k and v, cos / sin rows and the caller's
  // position and slot, copied by the lanes that own the row
  auto load_new_late = [&](int s0, int buf) {
    const int r = new_pos - s0;
    if (r % ROW_STEP == row0) {
      load_new_inputs(new_pos);
      const int64_t src = int64_t(b) * a.new_stride_b + int64_t(hk) * a.new_stride_h + part * 16;
      unsigned char* kdst = wbuf + buf * CF::kWarpStage + part * 16 + r * CF::kRowBytes;
      cp_async16(kdst, a.new_k + src, 16);
      cp_async16(kdst + CF::kStageBytes, a.new_v + src, 16);
    }
    cp_async_commit();
  };

  // warp w takes stages w, w + W, w + 2W, ... of the chunk
  const int n_stages = (tok1 - tok0 + kStageTok - 1) / kStageTok;
  const int n_my = warp < n_stages ? (n_stages - warp + W - 1) / W : 0;
  const bool round_twice = DT == AUGUR_KV_F16 || !a.scale_exact;
  // scores to base 2: one multiply when no second rounding sits between the
  // division by sqrt(head_dim) and the change of base
  const float scale1 = round_twice ? (a.scale_exact ? a.inv_sqrt_d : 1.f) : a.inv_sqrt_d * kLog2e;
  const int mat = lane >> 3, r8 = lane & 7;
  // stage i of this warp starts at token tok0 + (warp + i W) * 32; the first
  // NS stages load up front, and each buffer refills as soon as it is computed
  auto load_first = [&](bool late) {
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      if (i < n_my) load_stage(tok0 + (warp + i * W) * kStageTok, i, late);
      else cp_async_commit();
    }
  };
  // early reads: the new token of a fused launch (its k / v come from the
  // previous kernel) is copied after the wait. With one stage buffer per
  // warp only its row waits; with more, the warp's first stages do.
  bool defer = false, late_new = false;
  if (FUSE && early && first_item) {
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      const int s0 = tok0 + (warp + i * W) * kStageTok;
      const bool has = i < n_my && new_pos >= s0 && new_pos < s0 + kStageTok;
      if (NS == 1) late_new = late_new || has;
      else defer = defer || has;
    }
  }
  if (!defer) load_first(late_new);
  if (first_item) {
    if (early) asm volatile("griddepcontrol.wait;" ::: "memory");
    // this CTA's first loads are issued (and the previous kernel is done):
    // the next kernel may start launching
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    first_item = false;
  }
  if (defer) load_first(false);
  if (late_new) load_new_late(tok0 + warp * kStageTok, 0);  // one stage buffer: its row 0 stage
  // Q^T as mma B fragments: b0 = Q[head nt*8+g][dims ks*16+2t, +1], b1 the
  // same 8 dims further (heads >= G are 0).
  {
    const char* qbase = a.q + int64_t(b) * a.q_stride_b;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int head = nt * 8 + g;
      const char* qrow = qbase + int64_t(hk * G + head) * a.q_stride_h;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t v0 = 0, v1 = 0;
        if (head < G) {
          v0 = *reinterpret_cast<const uint32_t*>(qrow + (ks * 16 + 2 * t) * 2);
          v1 = *reinterpret_cast<const uint32_t*>(qrow + (ks * 16 + 8 + 2 * t) * 2);
        }
        qb[ks][nt][0] = v0;
        qb[ks][nt][1] = v1;
      }
    }
  }

  if (warp == 0) publish(slot ^ 1, next_id());  // overlaps this warp's loads
  if (FUSE && n_my > 0 && S > 0) {
    // fused launches: q arrives before RoPE. Dims d and d + D/2 of a head sit
    // in the same lane (k-steps ks and ks + D/32), so each lane rotates its
    // own fragments with the new token's cos / sin row.
    const int pos = S - 1;
    if (pos < a.rope_n) {
      const char* cs = a.rope_cos + int64_t(pos) * D;
      const char* sn = a.rope_sin + int64_t(pos) * D;
#pragma unroll
      for (int ks = 0; ks < D / 32; ++ks) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int dim = ks * 16 + j * 8 + 2 * t;
          const uint32_t cv = *reinterpret_cast<const uint32_t*>(cs + dim * 2);
          const uint32_t sv = *reinterpret_cast<const uint32_t*>(sn + dim * 2);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) rope_pair<T>(qb[ks][nt][j], qb[ks + D / 32][nt][j], cv, sv);
        }
      }
    }
  }
  for (int it = 0; it < n_my; ++it) {
    const int s0 = tok0 + (warp + it * W) * kStageTok;
    cp_async_wait<NS - 1>();
    __syncwarp();
    const unsigned char* Ks = wbuf + (it % NS) * CF::kWarpStage;
    const unsigned char* Vs = Ks + CF::kStageBytes;
    if (FUSE && new_pos >= s0 && new_pos < s0 + kStageTok) {
      // fused launches: the new token's row holds its k and v as given; rotate
      // k in place (lane l: pieces l and l + PARTS/2, the two halves of the
      // row) and write the rotated k and the v to the token's pool row
      unsigned char* kr = const_cast<unsigned char*>(Ks) + (new_pos - s0) * CF::kRowBytes;
      unsigned char* vr = const_cast<unsigned char*>(Vs) + (new_pos - s0) * CF::kRowBytes;
      const int64_t dofs = *new_ofs;
      if (lane == 0 && a.chk_pos != nullptr && (new_chk[0] != int64_t(new_pos) || new_chk[1] != new_chk[2]))
        record_status(a.status, AUGUR_KV_EBOUNDS);  // the caller's position or slot is not the table's
      if (lane < PARTS / 2) {
        uint4 x1 = *reinterpret_cast<const uint4*>(kr + lane * 16);
        uint4 x2 = *reinterpret_cast<const uint4*>(kr + (lane + PARTS / 2) * 16);
        const uint4 cv = *reinterpret_cast<const uint4*>(new_cs + lane * 16);
        const uint4 sv = *reinterpret_cast<const uint4*>(new_sn + lane * 16);
        rope_pair<T>(x1.x, x2.x, cv.x, sv.x);
        rope_pair<T>(x1.y, x2.y, cv.y, sv.y);
        rope_pair<T>(x1.z, x2.z, cv.z, sv.z);
        rope_pair<T>(x1.w, x2.w, cv.w, sv.w);
        *reinterpret_cast<uint4*>(kr + lane * 16) = x1;
        *reinterpret_cast<uint4*>(kr + (lane + PARTS / 2) * 16) = x2;
        if (dofs >= 0) {
          *reinterpret_cast<uint4*>(a.k_w + dofs + lane * 16) = x1;
          *reinterpret_cast<uint4*>(a.k_w + dofs + (lane + PARTS / 2) * 16) = x2;
        }
      }
      if (lane < PARTS && dofs >= 0)
        *reinterpret_cast<uint4*>(a.v_w + dofs + lane * 16) = *reinterpret_cast<const uint4*>(vr + lane * 16);
      __syncwarp();
    }

    // S^T: two 16-token row tiles x NT 8-head column tiles
    float s[2][NT][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) s[mt][nt][0] = s[mt][nt][1] = s[mt][nt][2] = s[mt][nt][3] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int tok = mt * 16 + (mat & 1) * 8 + r8;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t ka[4];
        ldmatrix_x4(ka, Ks + tok * CF::kRowBytes + (ks * 16 + (mat >> 1) * 8) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<T>(s[mt][nt], ka, qb[ks][nt][0], qb[ks][nt][1]);
      }
    }
    // round as the reference's dtype matmul and scalar division do, move to
    // base 2, mask the tail of the last stage (rows are tokens)
    const bool full = s0 + kStageTok <= tok1;
    // one loop body per rounding mode, chosen once per stage (warp-uniform)
    auto scores = [&](auto twice, auto divide) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
          const bool dead = !full && s0 + mt * 16 + hp * 8 + g >= tok1;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            float2 r = round2<T>(s[mt][nt][2 * hp], s[mt][nt][2 * hp + 1]);
            float x0, x1;
            if constexpr (decltype(twice)::value) {
              if constexpr (decltype(divide)::value) {
                r.x /= a.sqrt_d;
                r.y /= a.sqrt_d;
              } else {
                r.x *= scale1;
                r.y *= scale1;
              }
              r = round2<T>(r.x, r.y);
              x0 = r.x * kLog2e;
              x1 = r.y * kLog2e;
            } else {
              x0 = r.x * scale1;
              x1 = r.y * scale1;
            }
            s[mt][nt][2 * hp] = dead ? kNegInf : x0;
            s[mt][nt][2 * hp + 1] = dead ? kNegInf : x1;
          }
        }
      }
    };
    if (!round_twice) scores(std::false_type{}, std::false_type{});
    else if (a.scale_exact) scores(std::true_type{}, std::false_type{});
    else scores(std::true_type{}, std::true_type{});
    // column (head) maxima over the stage's 32 tokens: this lane's 4, then the 8 g-lanes
    float mnew[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float m = fmaxf(fmaxf(s[0][nt][j], s[0][nt][2 + j]), fmaxf(s[1][nt][j], s[1][nt][2 + j]));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        mnew[nt][j] = fmaxf(mrow[nt][j], m);  // finite: every stage holds a valid token
      }
    }
    if (it > 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float al = ex2(mrow[nt][j] - mnew[nt][j]);
          lrow[nt][j] *= al;
#pragma unroll
          for (int dm = 0; dm < D / 16; ++dm) {
            o[dm][nt][j] *= al;
            o[dm][nt][2 + j] *= al;
          }
        }
      }
    }
    // probabilities, rounded to the dtype, as P^T B fragments (movmatrix
    // turns the [token][head pair] layout of S^T into [head][token pair])
    uint32_t pb[2][NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      mrow[nt][0] = mnew[nt][0];
      mrow[nt][1] = mnew[nt][1];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float p0 = ex2(s[mt][nt][0] - mnew[nt][0]), p1 = ex2(s[mt][nt][1] - mnew[nt][1]);
        const float p2 = ex2(s[mt][nt][2] - mnew[nt][0]), p3 = ex2(s[mt][nt][3] - mnew[nt][1]);
        lrow[nt][0] += p0 + p2;
        lrow[nt][1] += p1 + p3;
        pb[mt][nt][0] = movmatrix_trans(pack2<T>(p0, p1));
        pb[mt][nt][1] = movmatrix_trans(pack2<T>(p2, p3));
      }
    }
    // O^T += V^T P^T: 16-dim row tiles, 16-token k-steps
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int tok = mt * 16 + (mat >> 1) * 8 + r8;
#pragma unroll
      for (int dm = 0; dm < D / 16; ++dm) {
        uint32_t va[4];
        ldmatrix_x4_trans(va, Vs + tok * CF::kRowBytes + (dm * 16 + (mat & 1) * 8) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<T>(o[dm][nt], va, pb[mt][nt][0], pb[mt][nt][1]);
      }
    }
    __syncwarp();  // every lane is done with the buffer before it is refilled
    const int nxt = it + NS;
    if (nxt < n_my) load_stage(tok0 + (warp + nxt * W) * kStageTok, nxt % NS, false);
    else cp_async_commit();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      lrow[nt][j] += __shfl_xor_sync(0xffffffffu, lrow[nt][j], 4);
      lrow[nt][j] += __shfl_xor_sync(0xffffffffu, lrow[nt][j], 8);
      lrow[nt][j] += __shfl_xor_sync(0xffffffffu, lrow[nt][j], 16);
    }
  }
  // warp -> its own stage buffer, which no other warp touches: [16 heads][PO]
  // partial outputs (the stores transpose O^T back), then 16 maxima, 16 sums
  {
    float* wp = reinterpret_cast<float*>(wbuf);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int dm = 0; dm < D / 16; ++dm) {
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          const int head = nt * 8 + 2 * t + (f & 1), dim = dm * 16 + g + (f >> 1) * 8;
          wp[head * PO + dim] = o[dm][nt][f];
        }
      }
      if (g == 0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          wp[16 * PO + nt * 8 + 2 * t + j] = mrow[nt][j];
          wp[16 * PO + 16 + nt * 8 + 2 * t + j] = lrow[nt][j];
        }
      }
    }
  }
  __syncthreads();
  if (int(threadIdx.x) < G) {
    const int row = threadIdx.x;
    float M = kNegInf;
    for (int w = 0; w < W; ++w) M = fmaxf(M, wpart[w * WSF + 16 * PO + row]);
    float L = 0.f;
    for (int w = 0; w < W; ++w) {
      const float mw = wpart[w * WSF + 16 * PO + row];
      const float f = mw == kNegInf ? 0.f : ex2(mw - M);
      fac[w * 16 + row] = f;
      L += wpart[w * WSF + 16 * PO + 16 + row] * f;
    }
    cta_m[row] = M;
    cta_l[row] = L;
  }
  __syncthreads();
  const int GD = G * D;
  char* ob = a.out + int64_t(b) * a.out_stride_b;
  if (my_nch == 1) {  // the whole sequence is in this CTA
    for (int i = threadIdx.x; i < GD; i += blockDim.x) {
      const int row = i / D, d = i - row * D;
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) O += wpart[w * WSF + row * PO + d] * fac[w * 16 + row];
      const float L = cta_l[row];
      store_elem(ob + int64_t(hk * G + row) * a.out_stride_h + d * 2, DT, L > 0.f ? O / L : 0.f);
    }
    continue;
  }
  // partial of this chunk -> the scratch slot of this item
  float* wo = a.ws_o + int64_t(item_first) * GD;
  float* wml = a.ws_ml + int64_t(item_first) * 32;
  for (int i = threadIdx.x; i < GD; i += blockDim.x) {
    const int row = i / D, d = i - row * D;
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) O += wpart[w * WSF + row * PO + d] * fac[w * 16 + row];
    wo[int64_t(chunk) * GD + i] = O;
  }
  if (int(threadIdx.x) < G) {
    wml[chunk * 32 + threadIdx.x] = cta_m[threadIdx.x];
    wml[chunk * 32 + 16 + threadIdx.x] = cta_l[threadIdx.x];
  }
  const int64_t unit = int64_t(b) * a.hkv + hk;
  // One release-acquire increment by thread 0 after the barrier publishes the
  // whole CTA's partial (barrier then release is cumulative) and, for the
  // last CTA, makes every other CTA's partial visible to the reads below.
  __syncthreads();
  if (threadIdx.x == 0) *last_flag = atom_add_acq_rel_gpu(a.ws_cnt + unit, 1) == my_nch - 1;
  __syncthreads();
  if (!*last_flag) continue;
  // last CTA of the (sequence, KV head): combine every chunk's partial. The
  // row maxima and sums of all chunks and (for up to kCombineRegs chunks)
  // this thread's partial outputs load together, in one round of requests.
  constexpr int kPerThread = (NT * 8 * D + CF::kThreads - 1) / CF::kThreads;  // outputs per thread
  constexpr int kCombineRegs = AUGUR_KV_ATTN_COMBINE_REGS / kPerThread > 1 ? AUGUR_KV_ATTN_COMBINE_REGS / kPerThread : 1;
  float* cm = reinterpret_cast<float*>(smem);  // [my_nch][16] maxima, then rescale factors
  float* cl = cm + kMaxChunks * 16;            // [my_nch][16] sums
  float pv[kPerThread][kCombineRegs];
  const bool in_regs = my_nch <= kCombineRegs;
  if (in_regs) {
#pragma unroll
    for (int e = 0; e < kPerThread; ++e) {
      const int i = threadIdx.x + e * CF::kThreads;
#pragma unroll
      for (int c = 0; c < kCombineRegs; ++c)
        pv[e][c] = (i < GD && c < my_nch) ? __ldcg(wo + int64_t(c) * GD + i) : 0.f;
    }
  }
  for (int j = threadIdx.x; j < my_nch * G; j += blockDim.x) {
    const int c = j / G, row = j - c * G;
    cm[c * 16 + row] = __ldcg(wml + c * 32 + row);
    cl[c * 16 + row] = __ldcg(wml + c * 32 + 16 + row);
  }
  __syncthreads();
  if (int(threadIdx.x) < G) {
    const int row = threadIdx.x;
    float M = kNegInf;
    for (int c = 0; c < my_nch; ++c) M = fmaxf(M, cm[c * 16 + row]);
    float L = 0.f;
    for (int c = 0; c < my_nch; ++c) {
      const float mc = cm[c * 16 + row];
      const float f = mc == kNegInf ? 0.f : ex2(mc - M);
      cm[c * 16 + row] = f;
      L += cl[c * 16 + row] * f;
    }
    cta_l[row] = L;
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kPerThread; ++e) {
    const int i = threadIdx.x + e * CF::kThreads;
    if (i < GD) {
      const int row = i / D, d = i - row * D;
      float O = 0.f;
      if (in_regs) {
#pragma unroll
        for (int c = 0; c < kCombineRegs; ++c)
          if (c < my_nch) O += pv[e][c] * cm[c * 16 + row];
      } else {
#pragma unroll 8
        for (int c = 0; c < my_nch; ++c) O += __ldcg(wo + int64_t(c) * GD + i) * cm[c * 16 + row];
      }
      const float L = cta_l[row];
      store_elem(ob + int64_t(hk * G + row) * a.out_stride_h + d * 2, DT, L > 0.f ? O / L : 0.f);
    }
  }
  if (threadIdx.x == 0) a.ws_cnt[unit] = 0;  // ready for the next launch
  }  // items
}

// ---------------------------------------------------------------------------
// Generic path: one CTA per (sequence, query head), the reference's order
// ---------------------------------------------------------------------------

constexpr int kGenericThreads = 128;

__global__ void __launch_bounds__(kGenericThreads) attn_decode_generic_kernel(AttnArgs a) {
  extern __shared__ __align__(16) float gsm[];
  float* qv = gsm;                      // head_dim
  float* red = qv + a.head_dim;         // kGenericThreads
  float* sc = red + kGenericThreads;    // max_seq scores
  const int hq = blockIdx.x, b = blockIdx.y;
  const int hk = hq / a.groups;
  const int S = min(max(0, __ldg(a.seq_lens + b)), a.max_seq);
  const int D = a.head_dim;
  const int es = elem_size_dev(a.dtype);
  const char* qrow = a.q + int64_t(b) * a.q_stride_b + int64_t(hq) * a.q_stride_h;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qv[d] = load_elem(qrow + int64_t(d) * es, a.dtype);
  __syncthreads();

  // scores, rounded as the reference's dtype matmul and division round them
  float local_max = kNegInf;
  for (int pos = threadIdx.x; pos < S; pos += blockDim.x) {
    const char* kr = row_addr(a, a.k, b, hk, pos);
    float x = kNegInf;
    if (kr != nullptr) {
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(qv[d], load_elem(kr + int64_t(d) * es, a.dtype), acc);
      x = round_to(round_to(acc, a.dtype) / a.sqrt_d, a.dtype);
    }
    sc[pos] = x;
    local_max = fmaxf(local_max, x);
  }
  red[threadIdx.x] = local_max;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (int(threadIdx.x) < w) red[threadIdx.x] = fmaxf(red[threadIdx.x], red[threadIdx.x + w]);
    __syncthreads();
  }
  const float M = red[0];
  __syncthreads();
  float local_sum = 0.f;
  for (int pos = threadIdx.x; pos < S; pos += blockDim.x) {
    const float e = (sc[pos] == kNegInf || M == kNegInf) ? 0.f : expf(sc[pos] - M);
    sc[pos] = e;
    local_sum += e;
  }
  red[threadIdx.x] = local_sum;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (int(threadIdx.x) < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  const float L = red[0];
  __syncthreads();
  // probabilities in float32, cast to the dtype, then P.V accumulated in float32
  for (int pos = threadIdx.x; pos < S; pos += blockDim.x) sc[pos] = L > 0.f ? round_to(sc[pos] / L, a.dtype) : 0.f;
  __syncthreads();
  char* orow = a.out + int64_t(b) * a.out_stride_b + int64_t(hq) * a.out_stride_h;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int pos = 0; pos < S; ++pos) {
      const char* vr = row_addr(a, a.v, b, hk, pos);
      if (vr != nullptr) acc = fmaf(sc[pos], load_elem(vr + int64_t(d) * es, a.dtype), acc);
    }
    store_elem(orow + int64_t(d) * es, a.dtype, acc);
  }
}

}  // namespace augur_kv_dev

using namespace augur_kv_dev;

#define AUGUR_KV_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Launch shape of the split kernel: a persistent grid of the resident CTAs
// (slots). The kernel picks its chunk size on the device (never below
// chunk_min) so its work items number at most kItemWaves x slots.
// Counters (zero before the first launch, left zero by every launch, never
// used for data, so launches of any size may share them): two scheduler words
// padded to 256 bytes, then one arrival counter per (sequence, KV head) unit
// when a sequence can split. Scratch (no initial contents), indexed by work
// item: max_items x 32 floats (row maxima and sums), then max_items x G x D
// partial outputs; none when no sequence can split.
#ifndef AUGUR_KV_ATTN_ITEM_WAVES
#define AUGUR_KV_ATTN_ITEM_WAVES 4
#endif
constexpr int kItemWaves = AUGUR_KV_ATTN_ITEM_WAVES;
constexpr int64_t kSchedBytes = 256;

struct SplitPlan {
  int chunk_min = 0, max_items = 0;
  int64_t grid = 0, cnt_bytes = 0, ml_bytes = 0, scratch_bytes = 0;
};

SplitPlan plan_split(int batch, int hkv, int G, int D, int max_seq, int slots, int unit) {
  SplitPlan p;
  int64_t C = unit;
  while ((int64_t(max_seq) + C - 1) / C > kMaxChunks) C *= 2;
  p.chunk_min = int(C);
  p.grid = slots;
  p.max_items = kItemWaves * slots;
  const int64_t units = int64_t(batch) * hkv;
  p.cnt_bytes = kSchedBytes;
  if (units <= p.max_items && max_seq > C) {
    p.cnt_bytes += units * 4;
    p.ml_bytes = align256(int64_t(p.max_items) * 32 * 4);
    p.scratch_bytes = p.ml_bytes + int64_t(p.max_items) * G * D * 4;
  }
  return p;
}

bool mma_shape_ok(int dtype, int head_dim, int groups) {
  return dtype != AUGUR_KV_F32 && (head_dim == 64 || head_dim == 128) && groups <= 16;
}

// Resident CTAs of one split-kernel instance on the current device (cached).
template <typename T, int D, int NT, int NS>
int split_slots(int* slots_out) {
  using CF = SplitCfg<D, NS>;
  auto kern = attn_decode_split_kernel<T, D, NT, NS, false>;
  auto kern_fused = attn_decode_split_kernel<T, D, NT, NS, true>;
  static int slots[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(AUGUR_KV_ECUDA, "paged_decode_attention: cannot query the current device");
  const int sms = sm_count();
  std::lock_guard<std::recursive_mutex> lock(g_cache_mutex);
  if (slots[dev] == 0) {
    int per_sm = 0;
    int per_sm_fused = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kBytes) != cudaSuccess ||
        cudaFuncSetAttribute(kern_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kBytes) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, CF::kThreads, CF::kBytes) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_fused, kern_fused, CF::kThreads, CF::kBytes) !=
            cudaSuccess)
      return check_launch("attn_decode_split_kernel occupancy");
    // one grid size for both (the persistent grid must be resident either way)
    slots[dev] = std::max(1, std::min(per_sm, per_sm_fused)) * sms;
  }
  *slots_out = slots[dev];
  return AUGUR_KV_OK;
}

template <typename T, int D, int NT, int NS>
int launch_split(AttnArgs a, int max_seq, int32_t* cnt, int64_t cnt_bytes, void* scratch, int64_t scratch_bytes,
                 cudaStream_t st) {
  using CF = SplitCfg<D, NS>;
  int slots = 0;
  const int rc = split_slots<T, D, NT, NS>(&slots);
  if (rc != AUGUR_KV_OK) return rc;
  const SplitPlan p = plan_split(a.batch, a.hkv, a.groups, D, max_seq, slots, CF::kChunkUnit);
  a.chunk = p.chunk_min;
  a.max_items = p.max_items;
  if (cnt != nullptr && cnt_bytes >= kSchedBytes) a.ws_sched = cnt;  // dynamic item scheduling
  if (p.scratch_bytes > 0 && cnt != nullptr && cnt_bytes >= p.cnt_bytes && scratch != nullptr &&
      scratch_bytes >= p.scratch_bytes) {
    a.ws_cnt = cnt + kSchedBytes / 4;
    a.ws_ml = static_cast<float*>(scratch);
    a.ws_o = reinterpret_cast<float*>(static_cast<char*>(scratch) + p.ml_bytes);
  } else {
    // no room to combine chunks: one chunk per sequence (chunk sizes stay powers of two)
    int64_t C = CF::kChunkUnit;
    while (C < max_seq) C *= 2;
    a.chunk = int(C);
  }
  // programmatic dependent launch: the CTAs may become resident while the
  // previous kernel drains; the kernel waits for it before reading anything
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(unsigned(p.grid), 1, 1);
  cfg.blockDim = dim3(CF::kThreads, 1, 1);
  cfg.dynamicSmemBytes = CF::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = a.fuse ? cudaLaunchKernelEx(&cfg, attn_decode_split_kernel<T, D, NT, NS, true>, a)
                               : cudaLaunchKernelEx(&cfg, attn_decode_split_kernel<T, D, NT, NS, false>, a);
  if (e != cudaSuccess) return fail(AUGUR_KV_ECUDA, "attn_decode_split_kernel: %s", cudaGetErrorString(e));
  return check_launch("attn_decode_split_kernel");
}

template <typename T, int D, int NT, int NS>
int split_workspace(int batch, int hkv, int G, int max_seq, int64_t* cnt_bytes, int64_t* scratch_bytes) {
  int slots = 0;
  const int rc = split_slots<T, D, NT, NS>(&slots);
  if (rc != AUGUR_KV_OK) return rc;
  const SplitPlan p = plan_split(batch, hkv, G, D, max_seq, slots, SplitCfg<D, NS>::kChunkUnit);
  *cnt_bytes = p.cnt_bytes;
  *scratch_bytes = p.scratch_bytes;
  return AUGUR_KV_OK;
}

template <typename T, int D>
int launch_split_g(const AttnArgs& a, int max_seq, int32_t* cnt, int64_t cnt_bytes, void* scratch,
                   int64_t scratch_bytes, cudaStream_t st) {
  constexpr int NS = D == 64 ? AUGUR_KV_ATTN_STAGES : 1;
  return a.groups <= 8 ? launch_split<T, D, 1, NS>(a, max_seq, cnt, cnt_bytes, scratch, scratch_bytes, st)
                       : launch_split<T, D, 2, NS>(a, max_seq, cnt, cnt_bytes, scratch, scratch_bytes, st);
}

template <typename T, int D>
int split_workspace_g(int batch, int hkv, int G, int max_seq, int64_t* cnt_bytes, int64_t* scratch_bytes) {
  constexpr int NS = D == 64 ? AUGUR_KV_ATTN_STAGES : 1;
  return G <= 8 ? split_workspace<T, D, 1, NS>(batch, hkv, G, max_seq, cnt_bytes, scratch_bytes)
                : split_workspace<T, D, 2, NS>(batch, hkv, G, max_seq, cnt_bytes, scratch_bytes);
}

}  // namespace

AUGUR_KV_EXPORT int augur_kv_paged_decode_attention_workspace(int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                                                              int32_t head_dim, int32_t max_seq_len, int32_t dtype,
                                                              int32_t flags, int64_t* counters_bytes,
                                                              int64_t* scratch_bytes) {
  g_last_error[0] = '\0';
  if (counters_bytes == nullptr || scratch_bytes == nullptr)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention_workspace: null pointer argument");
  *counters_bytes = 0;
  *scratch_bytes = 0;
  if (elem_size(dtype) == 0 || batch < 0 || max_seq_len < 0 || n_q_heads <= 0 || n_kv_heads <= 0 ||
      n_q_heads % n_kv_heads != 0 || head_dim <= 0)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention_workspace: bad sizes");
  const int G = n_q_heads / n_kv_heads;
  if (batch == 0 || (flags & ~AUGUR_KV_ATTN_EARLY_READS) == AUGUR_KV_ATTN_GENERIC || !mma_shape_ok(dtype, head_dim, G))
    return AUGUR_KV_OK;
  if (max_seq_len > kMaxSeq)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention_workspace: max_seq_len above %d", kMaxSeq);
  if (dtype == AUGUR_KV_BF16)
    return head_dim == 64
               ? split_workspace_g<__nv_bfloat16, 64>(batch, n_kv_heads, G, max_seq_len, counters_bytes, scratch_bytes)
               : split_workspace_g<__nv_bfloat16, 128>(batch, n_kv_heads, G, max_seq_len, counters_bytes,
                                                       scratch_bytes);
  return head_dim == 64 ? split_workspace_g<__half, 64>(batch, n_kv_heads, G, max_seq_len, counters_bytes, scratch_bytes)
                        : split_workspace_g<__half, 128>(batch, n_kv_heads, G, max_seq_len, counters_bytes,
                                                         scratch_bytes);
}

namespace augur_kv_dev {

int paged_decode_attention_impl(
    const void* q, const int64_t* q_strides, const void* k_pool, const void* v_pool, const int64_t* pool_strides,
    int64_t num_blocks, int32_t block_size, const int32_t* block_tables, int64_t tables_stride, int64_t max_blocks,
    const int32_t* seq_lens, int32_t max_seq_len, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
    int32_t head_dim, int32_t dtype, void* out, const int64_t* out_strides, int32_t flags, int32_t* counters,
    int64_t counters_bytes, void* scratch, int64_t scratch_bytes, int32_t* status, void* stream, const FusedRope* fuse,
    bool* fused) {
  if (fused != nullptr) *fused = false;
  g_last_error[0] = '\0';
  const int es = elem_size(dtype);
  if (es == 0) return fail(AUGUR_KV_EINVAL, "paged_decode_attention: unknown dtype %d", dtype);
  if (batch < 0 || max_seq_len < 0) return fail(AUGUR_KV_EINVAL, "paged_decode_attention: negative sizes");
  if (batch == 0) return AUGUR_KV_OK;
  if (q == nullptr || k_pool == nullptr || v_pool == nullptr || pool_strides == nullptr || q_strides == nullptr ||
      block_tables == nullptr || seq_lens == nullptr || out == nullptr || out_strides == nullptr)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention: null pointer argument");
  if (n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks <= 0 || max_blocks <= 0 || batch > 65535 || n_kv_heads > 65535)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention: bad sizes");
  const int32_t kind = flags & ~AUGUR_KV_ATTN_EARLY_READS;
  if (kind < AUGUR_KV_ATTN_AUTO || kind > AUGUR_KV_ATTN_GENERIC)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention: unknown flags %d", flags);

  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.q = static_cast<const char*>(q);
  a.q_stride_b = q_strides[0] * es;
  a.q_stride_h = q_strides[1] * es;
  a.k = static_cast<const char*>(k_pool);
  a.v = static_cast<const char*>(v_pool);
  a.blk_stride = pool_strides[0] * es;
  a.head_stride = pool_strides[1] * es;
  a.row_stride = pool_strides[2] * es;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.tables = block_tables;
  a.tables_stride = tables_stride;
  a.max_blocks = max_blocks;
  a.seq_lens = seq_lens;
  a.batch = batch;
  a.hq = n_q_heads;
  a.hkv = n_kv_heads;
  a.groups = n_q_heads / n_kv_heads;
  a.head_dim = head_dim;
  a.sqrt_d = sqrtf(float(head_dim));
  {
    int e = 0;
    a.scale_exact = frexpf(a.sqrt_d, &e) == 0.5f ? 1 : 0;  // power of two: x * (1/s) == x / s
    a.inv_sqrt_d = 1.0f / a.sqrt_d;
  }
  a.out = static_cast<char*>(out);
  a.out_stride_b = out_strides[0] * es;
  a.out_stride_h = out_strides[1] * es;
  a.dtype = dtype;
  a.status = status;
  a.early = (flags & AUGUR_KV_ATTN_EARLY_READS) != 0 ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  a.max_seq = max_seq_len;
  a.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz(unsigned(block_size)) : -1;
  if (counters_bytes < 0 || scratch_bytes < 0 || (reinterpret_cast<uintptr_t>(counters) & 3u) != 0 ||
      (reinterpret_cast<uintptr_t>(scratch) & 15u) != 0)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention: counters 4-byte and scratch 16-byte aligned, sizes >= 0");

  // The tensor-core path needs a 16-bit dtype, head_dim 64 or 128, at most 16
  // query heads per KV head, and 16-byte aligned rows.
  uintptr_t align = reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) |
                    uintptr_t(a.blk_stride) | uintptr_t(a.head_stride) | uintptr_t(a.row_stride) |
                    reinterpret_cast<uintptr_t>(q) | uintptr_t(a.q_stride_b) | uintptr_t(a.q_stride_h);
  const bool mma_ok = mma_shape_ok(dtype, head_dim, a.groups) && (align & 15u) == 0 &&
                      a.row_stride == int64_t(head_dim) * es;
  if (fuse != nullptr) {
    // the fused RoPE write rides on the tensor-core kernel only; otherwise
    // nothing is launched and the caller issues the two launches
    const uintptr_t falign = reinterpret_cast<uintptr_t>(fuse->new_k) | reinterpret_cast<uintptr_t>(fuse->new_v) |
                             uintptr_t(fuse->new_stride_b * es) | uintptr_t(fuse->new_stride_h * es) |
                             reinterpret_cast<uintptr_t>(fuse->cos) | reinterpret_cast<uintptr_t>(fuse->sin);
    if (kind == AUGUR_KV_ATTN_GENERIC || !mma_ok || (falign & 15u) != 0 || fuse->new_k == nullptr ||
        fuse->new_v == nullptr || fuse->cos == nullptr || fuse->sin == nullptr || fuse->n_pos <= 0 ||
        max_seq_len > kMaxSeq)
      return AUGUR_KV_OK;
    a.fuse = 1;
    a.new_k = static_cast<const char*>(fuse->new_k);
    a.new_v = static_cast<const char*>(fuse->new_v);
    a.new_stride_b = fuse->new_stride_b * es;
    a.new_stride_h = fuse->new_stride_h * es;
    a.rope_cos = static_cast<const char*>(fuse->cos);
    a.rope_sin = static_cast<const char*>(fuse->sin);
    a.rope_n = fuse->n_pos;
    a.chk_pos = fuse->positions;
    a.chk_slot = fuse->positions != nullptr ? fuse->slots : nullptr;
    if ((fuse->positions == nullptr) != (fuse->slots == nullptr) ||
        ((reinterpret_cast<uintptr_t>(fuse->positions) | reinterpret_cast<uintptr_t>(fuse->slots)) & 7u) != 0)
      return fail(AUGUR_KV_EINVAL, "decode_layer: positions and slots must both be given, 8-byte aligned");
    a.k_w = static_cast<char*>(const_cast<void*>(k_pool));
    a.v_w = static_cast<char*>(const_cast<void*>(v_pool));
    if (fused != nullptr) *fused = true;
  }
  if (kind != AUGUR_KV_ATTN_GENERIC && mma_ok) {
    if (max_seq_len > kMaxSeq)
      return fail(AUGUR_KV_EINVAL, "paged_decode_attention: max_seq_len above %d", kMaxSeq);
    if (dtype == AUGUR_KV_BF16)
      return head_dim == 64 ? launch_split_g<__nv_bfloat16, 64>(a, max_seq_len, counters, counters_bytes, scratch, scratch_bytes, st)
                            : launch_split_g<__nv_bfloat16, 128>(a, max_seq_len, counters, counters_bytes, scratch, scratch_bytes, st);
    return head_dim == 64 ? launch_split_g<__half, 64>(a, max_seq_len, counters, counters_bytes, scratch, scratch_bytes, st)
                          : launch_split_g<__half, 128>(a, max_seq_len, counters, counters_bytes, scratch, scratch_bytes, st);
  }

  // generic path: the whole sequence's scores live in shared memory
  const size_t smem = size_t(head_dim + kGenericThreads + max_seq_len) * sizeof(float);
  if (smem > 200 * 1024)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention: generic path limited to %d positions",
                int(200 * 1024 / sizeof(float)) - head_dim - kGenericThreads);
  {
    static int attr_bytes[kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return fail(AUGUR_KV_ECUDA, "paged_decode_attention: cannot query the current device");
    std::lock_guard<std::recursive_mutex> lock(g_cache_mutex);
    if (smem > 48 * 1024 && size_t(attr_bytes[dev]) < smem) {
      if (cudaFuncSetAttribute(attn_decode_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               int(200 * 1024)) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(attn_decode_generic_kernel)");
      attr_bytes[dev] = 200 * 1024;
    }
  }
  attn_decode_generic_kernel<<<dim3(unsigned(n_q_heads), unsigned(batch), 1u), kGenericThreads, smem, st>>>(a);
  return check_launch("attn_decode_generic_kernel");
}

}  // namespace augur_kv_dev

AUGUR_KV_EXPORT int augur_kv_paged_decode_attention(
    const void* q, const int64_t* q_strides, const void* k_pool, const void* v_pool, const int64_t* pool_strides,
    int64_t num_blocks, int32_t block_size, const int32_t* block_tables, int64_t tables_stride, int64_t max_blocks,
    const int32_t* seq_lens, int32_t max_seq_len, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
    int32_t head_dim, int32_t dtype, void* out, const int64_t* out_strides, int32_t flags, int32_t* counters,
    int64_t counters_bytes, void* scratch, int64_t scratch_bytes, int32_t* status, void* stream) {
  return augur_kv_dev::paged_decode_attention_impl(q, q_strides, k_pool, v_pool, pool_strides, num_blocks, block_size,
                                                   block_tables, tables_stride, max_blocks, seq_lens, max_seq_len,
                                                   batch, n_q_heads, n_kv_heads, head_dim, dtype, out, out_strides,
                                                   flags, counters, counters_bytes, scratch, scratch_bytes, status,
                                                   stream, nullptr, nullptr);
}
