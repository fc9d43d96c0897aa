// augur_prefill.cu — attention of a batch's new tokens over the paged pool
// (prefill, or the suffix of a prompt whose prefix blocks are already cached).
//
// augur's paged branch (augur/attention.py:53-86) writes a call's new K/V into
// the pool, gathers the whole sequence back with read_paged_kv (:72), repeats
// each KV head for its query heads (:75-76), and computes q k^T / sqrt(d) in
// the cache dtype, a causal mask with past_len = key_len - query_len
// (_causal_mask, :15-19), a float32 softmax cast back to the dtype, and P V
// (:78-86). With a prefix-cached prompt (blocks shared through the prefix
// index) the call's query tokens are only the suffix, at positions past_len ..
// key_len - 1, and they attend to the cached prefix as well as to themselves.
// Here one launch covers every sequence of a batch for one layer and reads the
// pool in place: query token i of a sequence with n query tokens and seq_len
// cached positions (its own included) sits at position seq_len - n + i and
// attends to positions [0, seq_len - n + i].
//
//  * attn_prefill_umma_kernel (bf16 / fp16, head_dim 64 or 128, at most 8
//    query heads per KV head, 16-byte aligned rows): the work on the
//    5th-generation tensor cores, accumulators in tensor memory (described at
//    the kernel).
//  * attn_prefill_mma_kernel (the same shapes when q / out rows are only
//    4-byte aligned, or on request; bf16 / fp16, head_dim 64 or 128, at most 8 query
//    heads per KV head): one CTA per (sequence, KV head, tile of 16 query
//    tokens), one warp per query head of the group. K and V stream through
//    shared memory 64 keys at a time (cp.async, three stage buffers, the
//    block-table entry looked up per row); S = Q K^T and O += P V run on
//    mma.sync m16n8k16 around an online softmax in base 2. Tiles are issued
//    longest first (the last tile of a sequence reads the most keys).
//  * attn_prefill_generic_kernel (any dtype and shape): one CTA per (query
//    token, query head), the token's scores in shared memory, then the
//    reference's order: max, exp, sum, normalise, cast, P V.
//
// Rounding follows the reference where it rounds (scores to the dtype after
// q k and after the division by sqrt(head_dim); probabilities to the dtype
// before P V; the output once); sums run in another order, so results agree
// within a floating-point tolerance.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <type_traits>

#include "augur_kv.h"
#include "common.cuh"

namespace augur_kv_pf {

using augur_kv_dev::record_status;

struct PrefillArgs {
  const char* q;
  int64_t q_stride_t, q_stride_h;  // bytes; head_dim contiguous
  const char* k;
  const char* v;
  int64_t blk_stride, head_stride, row_stride;  // bytes
  int64_t num_blocks;
  int32_t block_size, bs_shift;  // log2(block_size) or -1
  const int32_t* tables;
  int64_t tables_stride, max_blocks;
  const int32_t* seq_lens;
  const int32_t* q_starts;
  int32_t batch, max_q_len, max_seq, hq, hkv, groups, head_dim, dtype;
  float sqrt_d, inv_sqrt_d;
  int32_t scale_exact;  // sqrt(head_dim) is a power of two
  char* out;
  int64_t out_stride_t, out_stride_h;  // bytes
  int32_t* status;
};

constexpr float kNegInf = -INFINITY;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kQT = 16;     // query tokens per CTA (one mma row tile)
constexpr int kStages = 3;  // stage buffers
constexpr int kMaxGroups = 8;
// Keys per stage and the resident CTAs per SM the head_dim-64 kernel is
// compiled for (head_dim 128 is compiled for one: its accumulators need more
// than 128 registers).
// Measured on B200 (config-4 suffix prefill: 256 x 128 query tokens over
// 1,152 cached positions, bf16, head_dim 64, per layer): 64 keys with 2 CTAs
// 840 us (152 TFLOP/s); 32 keys with 3 CTAs (80 registers, spills) 895 us;
// 64 keys unbounded (165 registers, 1 CTA) 1,098 us; 32 keys unbounded
// (139 registers) 1,366 us.
#ifndef AUGUR_KV_PREFILL_KT
#define AUGUR_KV_PREFILL_KT 64
#endif
#ifndef AUGUR_KV_PREFILL_MIN_CTAS
#define AUGUR_KV_PREFILL_MIN_CTAS 2
#endif
constexpr int kKT = AUGUR_KV_PREFILL_KT;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  static constexpr int dtype = AUGUR_KV_BF16;
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 round2(float x, float y) {
    return __bfloat1622float2(__floats2bfloat162_rn(x, y));
  }
};
template <> struct Mma<__half> {
  static constexpr int dtype = AUGUR_KV_F16;
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 round2(float x, float y) { return __half22float2(__floats2half2_rn(x, y)); }
};

__device__ __forceinline__ float ex2(float x) {  // 2^x; ex2(-inf) = 0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The sequence's query tokens and its causal offset; false (and EBOUNDS) when
// the lengths the caller gave are inconsistent.
__device__ __forceinline__ bool seq_bounds(const PrefillArgs& a, int b, int& q0, int& n, int& past) {
  q0 = __ldg(a.q_starts + b);
  n = __ldg(a.q_starts + b + 1) - q0;
  const int S = __ldg(a.seq_lens + b);
  past = S - n;
  if (n < 0 || past < 0 || S > a.max_seq || n > a.max_q_len) {
    record_status(a.status, AUGUR_KV_EBOUNDS);
    return false;
  }
  return true;
}

// Address of K or V row `pos` of sequence b, KV head hk; nullptr (and
// EBOUNDS) for a block outside the table or the pool.
__device__ __forceinline__ const char* pool_row(const PrefillArgs& a, const char* pool, int b, int hk, int pos) {
  const int lb = a.bs_shift >= 0 ? (pos >> a.bs_shift) : pos / a.block_size;
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

template <int D>
struct PfCfg {
  static constexpr int kRowBytes = D * 2 + 16;  // padded: ldmatrix rows hit distinct banks
  static constexpr int kTileBytes = kKT * kRowBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K then V
  static constexpr int kBytes = kStages * kStageBytes;
  static constexpr int kParts = D * 2 / 16;  // 16-byte pieces per row
};

template <typename T, int D>
__global__ void __launch_bounds__(kMaxGroups * 32, D == 64 ? AUGUR_KV_PREFILL_MIN_CTAS : 1)
    attn_prefill_mma_kernel(PrefillArgs a) {
  using CF = PfCfg<D>;
  using M = Mma<T>;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile = int(gridDim.x) - 1 - int(blockIdx.x);  // longest tiles first
  const int b = blockIdx.y / a.hkv, hk = blockIdx.y - b * a.hkv;
  int q0, n, past;
  if (!seq_bounds(a, b, q0, n, past)) return;
  const int i0 = tile * kQT;
  if (i0 >= n) return;
  const int i1 = min(n, i0 + kQT);
  const int key_end = past + i1;  // keys [0, key_end)
  const int n_st = (key_end + kKT - 1) / kKT;
  const int qh = hk * a.groups + warp;

  // Q of this warp's head as mma A fragments: rows = the tile's 16 tokens
  uint32_t qa[D / 16][4];
  {
    const char* r0 = i0 + g < n ? a.q + int64_t(q0 + i0 + g) * a.q_stride_t + int64_t(qh) * a.q_stride_h : nullptr;
    const char* r1 =
        i0 + g + 8 < n ? a.q + int64_t(q0 + i0 + g + 8) * a.q_stride_t + int64_t(qh) * a.q_stride_h : nullptr;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int c0 = (ks * 16 + 2 * t) * 2, c1 = c0 + 16;
      qa[ks][0] = r0 ? *reinterpret_cast<const uint32_t*>(r0 + c0) : 0u;
      qa[ks][1] = r1 ? *reinterpret_cast<const uint32_t*>(r1 + c0) : 0u;
      qa[ks][2] = r0 ? *reinterpret_cast<const uint32_t*>(r0 + c1) : 0u;
      qa[ks][3] = r1 ? *reinterpret_cast<const uint32_t*>(r1 + c1) : 0u;
    }
  }

  // every thread of the CTA stages pieces of the K and V rows of keys
  // [s * 32, s * 32 + 32); keys past key_end (or in a bad block) read as zero
  auto load_stage = [&](int s, int buf) {
    unsigned char* base = smem + buf * CF::kStageBytes;
    constexpr int kPieces = kKT * CF::kParts * 2;
    for (int p = threadIdx.x; p < kPieces; p += blockDim.x) {
      const int kv = p / (kKT * CF::kParts);
      const int rest = p - kv * (kKT * CF::kParts);
      const int row = rest / CF::kParts, part = rest - row * CF::kParts;
      const int key = s * kKT + row;
      const char* src = kv ? a.v : a.k;
      int bytes = 0;
      if (key < key_end) {
        const char* r = pool_row(a, src, b, hk, key);
        if (r != nullptr) {
          src = r + part * 16;
          bytes = 16;
        }
      }
      cp_async16(base + kv * CF::kTileBytes + row * CF::kRowBytes + part * 16, src, bytes);
    }
  };

  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {kNegInf, kNegInf}, lrow[2] = {0.f, 0.f};
  const bool round_twice = M::dtype == AUGUR_KV_F16 || !a.scale_exact;
  const float scale1 = round_twice ? (a.scale_exact ? a.inv_sqrt_d : 1.f) : a.inv_sqrt_d * kLog2e;
  const int qp0 = past + i0 + g, qp1 = qp0 + 8;  // positions of rows g and g + 8
  const int mat = lane >> 3, r8 = lane & 7;

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < n_st) load_stage(s, s);
    cp_async_commit();
  }
  for (int s = 0; s < n_st; ++s) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // stage s has landed everywhere; every warp is done with stage s - 1
    {
      const int nx = s + kStages - 1;
      if (nx < n_st) load_stage(nx, nx % kStages);
      cp_async_commit();
    }
    const unsigned char* Ks = smem + (s % kStages) * CF::kStageBytes;
    const unsigned char* Vs = Ks + CF::kTileBytes;
    // S = Q K^T: 16 tokens x kKT keys, 8-key n-tiles
    constexpr int NJ = kKT / 8;
    float sc[NJ][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < NJ / 2; ++np) {
        uint32_t kb[4];
        ldsm_x4(kb, Ks + (np * 16 + (mat >> 1) * 8 + r8) * CF::kRowBytes + (ks * 16 + (mat & 1) * 8) * 2);
        M::run(sc[2 * np], qa[ks], kb[0], kb[1]);
        M::run(sc[2 * np + 1], qa[ks], kb[2], kb[3]);
      }
    }
    // round as the reference's dtype matmul and division do, to base 2; the causal
    // mask only where the stage's last key is past the tile's first query
    const bool need_mask = (s + 1) * kKT - 1 > past + i0;
    float rmax[2] = {kNegInf, kNegInf};
    // one loop body per rounding mode and mask case, chosen once per stage
    auto scores = [&](auto twice, auto divide, auto masked) {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
          float2 r = M::round2(sc[j][2 * hp], sc[j][2 * hp + 1]);
          float x0, x1;
          if constexpr (decltype(twice)::value) {
            if constexpr (decltype(divide)::value) {
              r.x /= a.sqrt_d;
              r.y /= a.sqrt_d;
            } else {
              r.x *= scale1;
              r.y *= scale1;
            }
            r = M::round2(r.x, r.y);
            x0 = r.x * kLog2e;
            x1 = r.y * kLog2e;
          } else {
            x0 = r.x * scale1;
            x1 = r.y * scale1;
          }
          if constexpr (decltype(masked)::value) {
            const int key = s * kKT + j * 8 + 2 * t;
            const int qp = hp ? qp1 : qp0;
            x0 = key > qp ? kNegInf : x0;
            x1 = key + 1 > qp ? kNegInf : x1;
          }
          sc[j][2 * hp] = x0;
          sc[j][2 * hp + 1] = x1;
          rmax[hp] = fmaxf(rmax[hp], fmaxf(x0, x1));
        }
      }
    };
    using yes = std::true_type;
    using no = std::false_type;
    if (!round_twice) {
      if (need_mask) scores(no{}, no{}, yes{});
      else scores(no{}, no{}, no{});
    } else if (a.scale_exact) {
      if (need_mask) scores(yes{}, no{}, yes{});
      else scores(yes{}, no{}, no{});
    } else {
      if (need_mask) scores(yes{}, yes{}, yes{});
      else scores(yes{}, yes{}, no{});
    }
    float alpha[2];
#pragma unroll
    for (int hp = 0; hp < 2; ++hp) {
      float m = rmax[hp];
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      const float mnew = fmaxf(mrow[hp], m);  // finite: stage 0 holds key 0, which every row sees
      alpha[hp] = ex2(mrow[hp] - mnew);       // 0 on the first stage (mrow = -inf)
      mrow[hp] = mnew;
      lrow[hp] *= alpha[hp];
    }
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // probabilities, rounded to the dtype, as A fragments of P (16-key k-steps)
    uint32_t pa[NJ / 2][4];
#pragma unroll
    for (int kk = 0; kk < NJ / 2; ++kk) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int j = 2 * kk + h2;
        const float p0 = ex2(sc[j][0] - mrow[0]), p1 = ex2(sc[j][1] - mrow[0]);
        const float p2 = ex2(sc[j][2] - mrow[1]), p3 = ex2(sc[j][3] - mrow[1]);
        lrow[0] += p0 + p1;
        lrow[1] += p2 + p3;
        pa[kk][2 * h2] = M::pack(p0, p1);
        pa[kk][2 * h2 + 1] = M::pack(p2, p3);
      }
    }
    // O += P V: V^T fragments by transposing loads, two 8-dim n-tiles per load
#pragma unroll
    for (int kk = 0; kk < NJ / 2; ++kk) {
#pragma unroll
      for (int dn = 0; dn < D / 8; dn += 2) {
        uint32_t vb[4];
        ldsm_x4_t(vb, Vs + (kk * 16 + (mat & 1) * 8 + r8) * CF::kRowBytes + (dn + (mat >> 1)) * 8 * 2);
        M::run(o[dn], pa[kk], vb[0], vb[1]);
        M::run(o[dn + 1], pa[kk], vb[2], vb[3]);
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int hp = 0; hp < 2; ++hp) {
    lrow[hp] += __shfl_xor_sync(0xffffffffu, lrow[hp], 1);
    lrow[hp] += __shfl_xor_sync(0xffffffffu, lrow[hp], 2);
  }
#pragma unroll
  for (int hp = 0; hp < 2; ++hp) {
    const int i = i0 + g + 8 * hp;
    if (i >= n) continue;
    const float inv = lrow[hp] > 0.f ? 1.f / lrow[hp] : 0.f;
    char* orow = a.out + int64_t(q0 + i) * a.out_stride_t + int64_t(qh) * a.out_stride_h;
#pragma unroll
    for (int j = 0; j < D / 8; ++j)
      *reinterpret_cast<uint32_t*>(orow + (j * 8 + 2 * t) * 2) = M::pack(o[j][2 * hp] * inv, o[j][2 * hp + 1] * inv);
  }
}

// ---------------------------------------------------------------------------
// tcgen05 path: the products on the 5th-generation tensor cores, accumulators
// in tensor memory
// ---------------------------------------------------------------------------
//
// One CTA (4 warps) per (sequence, KV head, tile of 16 query tokens). The MMA
// rows are 8 head slots x 16 tokens (row = slot * 16 + token; slots past the
// group and tokens past the sequence are zero rows, never stored), so warp w
// owns rows (tensor-memory lanes) 32w .. 32w + 31 and each thread one row.
// Per 64-key stage: one thread issues S = Q K^T into tensor memory (kind::f16,
// M = 128, N = 64, four K = 16 steps) and commits it to an mbarrier; every
// thread loads its row of S (tcgen05.ld), applies the reference's rounding,
// the causal mask and an online softmax in base 2 with no shuffles, and
// writes its row of P (the dtype) to shared memory; then one thread issues the
// stage's O = P V into a second tensor-memory region, which every thread
// loads and folds into its row of the output held in registers. Operands sit
// in shared memory in the no-swizzle core-matrix layout (8 rows x 16 bytes per
// core matrix): Q, K and P K-major, V MN-major as the pool stores it (its rows
// copy in as they are). K and V are staged with cp.async, two stage buffers.
// Every mbarrier wait is bounded (%globaltimer, 2 s); on expiry the CTA records
// AUGUR_KV_ETIMEOUT, frees its tensor memory and returns.

constexpr int kUKeys = 64;   // keys per stage
constexpr int kURows = 128;  // MMA rows: 8 head slots x 16 tokens
constexpr int kUKV = 3;      // K/V stage buffers
constexpr int kUP = 2;       // P buffers

template <int D>
struct UCfg {
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row of Q or K
  static constexpr int kQBytes = kURows * D * 2;
  static constexpr int kKVBytes = kUKeys * D * 2;  // one K or V stage
  static constexpr int kPBytes = kURows * kUKeys * 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;
  static constexpr int kV = kK + kUKV * kKVBytes;
  static constexpr int kP = kV + kUKV * kKVBytes;
  static constexpr int kRed = kP + kUP * kPBytes;  // [2][128] row maxima of the two halves, then [2][128] sums
  static constexpr int kBar = kRed + 4 * kURows * 4;  // mbarriers (S x 2, O), then the tensor-memory address
  static constexpr int kBytes = kBar + 64;
  static constexpr int kRowGroup = kChunks * 128;  // K-major Q / K: bytes between 8-row groups
  static constexpr int kVChunk = (kUKeys / 8) * 128;  // MN-major V: bytes between 8-dim chunks
  static constexpr uint32_t kCols = 256;  // S x 2 (64 columns each), then O (D columns)
  static constexpr int kMinCtas = D == 64 ? 2 : 1;  // shared memory: 96 KB / 160 KB per CTA
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Shared-memory matrix descriptor, no swizzle: start address, leading byte
// offset (between the two K chunks of a K-major step, or between K groups of
// an MN-major operand), stride byte offset (between 8-row groups, or between
// MN chunks), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(lbo >> 4) << 16) | (uint64_t(sbo >> 4) << 32) |
         (uint64_t(1) << 46);
}
// Instruction descriptor for kind::f16: f32 accumulator, A and B of the
// cache dtype (bf16 = 1, f16 = 0), A K-major, B K-major or MN-major, N, M.
template <typename T>
__host__ __device__ constexpr uint32_t umma_idesc(int n, bool b_mn_major) {
  return (1u << 4) | ((Mma<T>::dtype == AUGUR_KV_BF16 ? 1u : 0u) << 7) |
         ((Mma<T>::dtype == AUGUR_KV_BF16 ? 1u : 0u) << 10) | (uint32_t(b_mn_major) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(kURows >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with this parity to complete; false after 2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try(bar, parity)) {
    if (global_ns() - t0 > 2000000000ull) return false;
  }
  return true;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 32 consecutive 32-bit columns of this thread's tensor-memory lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

constexpr int kUThreads = 256;  // two threads per row: warps w and w + 4 share tensor-memory lanes 32 (w % 4) ..

template <typename T, int D>
__global__ void __launch_bounds__(kUThreads, UCfg<D>::kMinCtas) attn_prefill_umma_kernel(PrefillArgs a) {
  using U = UCfg<D>;
  using M = Mma<T>;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile = int(gridDim.x) - 1 - int(blockIdx.x);  // longest tiles first
  const int b = blockIdx.y / a.hkv, hk = blockIdx.y - b * a.hkv;
  int q0, n, past;
  if (!seq_bounds(a, b, q0, n, past)) return;
  const int i0 = tile * kQT;
  if (i0 >= n) return;
  const int i1 = min(n, i0 + kQT);
  const int key_end = past + i1;
  const int n_st = (key_end + kUKeys - 1) / kUKeys;
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + U::kBar);  // [2]: S buffers
  uint64_t* bar_o = bar_s + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + U::kBar + 32);
  const uint32_t sb = smem_u32(smem);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(U::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_s + 1, 1);
    mbar_init(bar_o, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Q: row r = slot * 16 + token, K-major core matrices
  for (int p = tid; p < kURows * U::kChunks; p += kUThreads) {
    const int r = p / U::kChunks, c = p - (p / U::kChunks) * U::kChunks;
    const int slot = r >> 4, tok = r & 15;
    const bool ok = slot < a.groups && i0 + tok < n;
    const char* src = ok ? a.q + int64_t(q0 + i0 + tok) * a.q_stride_t + int64_t(hk * a.groups + slot) * a.q_stride_h +
                               c * 16
                         : a.q;
    cp_async16(smem + U::kQ + (r >> 3) * U::kRowGroup + c * 128 + (r & 7) * 16, src, ok ? 16 : 0);
  }
  // K/V staging: 2 x 64 rows (K then V), each split into two halves of
  // kChunks / 2 pieces, one (K or V, row, half) per thread. A thread's
  // block-table entry for a stage is read one stage before its rows are
  // copied, so the copies never wait on the table.
  static_assert(2 * kUKeys * 2 == kUThreads, "one K/V half row per thread");
  constexpr int kHalfChunks = U::kChunks / 2;
  const int kv_sel = tid >= 2 * kUKeys;
  const int kv_row = (tid - kv_sel * 2 * kUKeys) >> 1, kv_c0 = (tid & 1) * kHalfChunks;
  const int32_t* kv_table = a.tables + int64_t(b) * a.tables_stride;
  // block id of this thread's key of stage s; -1: past the sequence; -2: past the table
  auto table_entry = [&](int s) -> int {
    const int key = s * kUKeys + kv_row;
    if (key >= key_end) return -1;
    const int lb = a.bs_shift >= 0 ? (key >> a.bs_shift) : key / a.block_size;
    return lb < a.max_blocks ? __ldg(kv_table + lb) : -2;
  };
  auto load_kv = [&](int s, int buf, int blk) {
    unsigned char* kd = smem + U::kK + buf * U::kKVBytes;
    unsigned char* vd = smem + U::kV + buf * U::kKVBytes;
    const int key = s * kUKeys + kv_row;
    const char* src = a.k;
    int bytes = 0;
    if (key < key_end) {
      if (blk >= 0 && blk < a.num_blocks) {
        const int lb = a.bs_shift >= 0 ? (key >> a.bs_shift) : key / a.block_size;
        src = (kv_sel ? a.v : a.k) + int64_t(blk) * a.blk_stride + int64_t(hk) * a.head_stride +
              int64_t(key - lb * a.block_size) * a.row_stride;
        bytes = 16;
      } else {
        record_status(a.status, AUGUR_KV_EBOUNDS);  // reads as zeros
      }
    }
#pragma unroll
    for (int c = kv_c0; c < kv_c0 + kHalfChunks; ++c) {
      unsigned char* dst = kv_sel ? vd + c * U::kVChunk + (kv_row >> 3) * 128 + (kv_row & 7) * 16
                                  : kd + (kv_row >> 3) * U::kRowGroup + c * 128 + (kv_row & 7) * 16;
      cp_async16(dst, src + (bytes ? c * 16 : 0), bytes);
    }
  };
  constexpr uint32_t idesc_s = umma_idesc<T>(kUKeys, false);
  constexpr uint32_t idesc_o = umma_idesc<T>(D, true);
  auto issue_s = [&](int s, uint32_t t_dst) {  // one thread: S_s = Q K_s^T, then arrive on bar_s[s & 1]
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks)
      umma_f16(t_dst, umma_desc(sb + U::kQ + ks * 256, 128, U::kRowGroup),
               umma_desc(sb + U::kK + (s % kUKV) * U::kKVBytes + ks * 256, 128, U::kRowGroup), idesc_s, ks > 0);
    umma_commit(bar_s + (s & 1));
  };
  load_kv(0, 0, table_entry(0));
  cp_async_commit();  // Q and stage 0
  if (n_st > 1) load_kv(1, 1, table_entry(1));
  cp_async_commit();  // stage 1
  int next_blk = n_st > 2 ? table_entry(2) : -1;  // for the stage loaded at the end of iteration 0
  cp_async_wait<1>();
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o = tmem + 2 * uint32_t(kUKeys);
  const int half = warp >> 2;  // this thread's 32 keys of each stage and D / 2 output dims
  const uint32_t my_lanes = uint32_t((warp & 3) * 32) << 16;
  if (tid == 0) issue_s(0, tmem);
  const int row = (warp & 3) * 32 + (tid & 31), slot = row >> 4, tok = row & 15;
  float* red_m = reinterpret_cast<float*>(smem + U::kRed);  // [2][128]
  float* red_l = red_m + 2 * kURows;                        // [2][128]
  const int qp = past + i0 + tok;
  const bool round_twice = M::dtype == AUGUR_KV_F16 || !a.scale_exact;
  const float scale1 = round_twice ? (a.scale_exact ? a.inv_sqrt_d : 1.f) : a.inv_sqrt_d * kLog2e;
  constexpr int DH = D / 2;  // output dims of this thread
  float o[DH];
#pragma unroll
  for (int d = 0; d < DH; ++d) o[d] = 0.f;
  float mrow = kNegInf, lrow = 0.f, alpha_prev = 0.f;
  bool ok = true;
  // fold the previous stage's P V (in tensor memory) into the output row
  auto fold = [&](int s_done) -> bool {
    if (!__syncthreads_and(tid != 0 || mbar_wait(bar_o, uint32_t(s_done) & 1u))) return false;
    tc_fence_after();
#pragma unroll
    for (int d0 = 0; d0 < DH; d0 += 32) {
      float h[32];
      tmem_ld32(t_o + my_lanes + half * DH + d0, h);
#pragma unroll
      for (int j = 0; j < 32; ++j) o[d0 + j] = o[d0 + j] * alpha_prev + h[j];
    }
    return true;
  };
  for (int s = 0; s < n_st; ++s) {
    // stage s + 1's rows have landed: its S goes to the tensor core while this
    // stage's softmax runs
    if (s + 1 < n_st) cp_async_wait<0>();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0 && s + 1 < n_st) issue_s(s + 1, tmem + uint32_t((s + 1) & 1) * kUKeys);
    // one thread waits on the mbarrier; the others sleep at the CTA barrier
    ok = __syncthreads_and(tid != 0 || mbar_wait(bar_s + (s & 1), uint32_t(s >> 1) & 1u));
    if (!ok) break;
    tc_fence_after();
    // this row's scores: round as the reference's dtype matmul and division do,
    // base 2, causal mask where the stage reaches past the tile's first query
    const bool need_mask = (s + 1) * kUKeys - 1 > past + i0;
    constexpr int KH = kUKeys / 2;  // this thread's keys of the stage
    float sv[KH];
    tmem_ld32(tmem + uint32_t(s & 1) * kUKeys + my_lanes + half * KH, sv);
    float mx = kNegInf;
    // one loop body per rounding mode, chosen once per stage (CTA-uniform), so
    // the unrolled loop issues only the mode's own instructions
    auto scores = [&](auto twice, auto divide, auto masked) {
#pragma unroll
      for (int j = 0; j < KH; j += 2) {
        float2 r = M::round2(sv[j], sv[j + 1]);
        float x0, x1;
        if constexpr (decltype(twice)::value) {
          if constexpr (decltype(divide)::value) {
            r.x /= a.sqrt_d;
            r.y /= a.sqrt_d;
          } else {
            r.x *= scale1;
            r.y *= scale1;
          }
          r = M::round2(r.x, r.y);
          x0 = r.x * kLog2e;
          x1 = r.y * kLog2e;
        } else {
          x0 = r.x * scale1;
          x1 = r.y * scale1;
        }
        if constexpr (decltype(masked)::value) {
          const int key = s * kUKeys + half * KH + j;
          x0 = key > qp ? kNegInf : x0;
          x1 = key + 1 > qp ? kNegInf : x1;
        }
        sv[j] = x0;
        sv[j + 1] = x1;
        mx = fmaxf(mx, fmaxf(x0, x1));
      }
    };
    using yes = std::true_type;
    using no = std::false_type;
    if (!round_twice) {
      if (need_mask) scores(no{}, no{}, yes{});
      else scores(no{}, no{}, no{});
    } else if (a.scale_exact) {
      if (need_mask) scores(yes{}, no{}, yes{});
      else scores(yes{}, no{}, no{});
    } else {
      if (need_mask) scores(yes{}, yes{}, yes{});
      else scores(yes{}, yes{}, no{});
    }
    // the row's maximum over both halves (red_m is rewritten only after the
    // next stage's first barrier, when both halves have read it)
    red_m[half * kURows + row] = mx;
    __syncthreads();
    mx = fmaxf(red_m[row], red_m[kURows + row]);
    const float mnew = fmaxf(mrow, mx);  // finite: stage 0 holds key 0, which every row sees
    const float alpha = ex2(mrow - mnew);
    mrow = mnew;
    lrow *= alpha;
    // P (the dtype) -> P buffer s & 1 (its last reader, P V of stage s - 2, is done)
    unsigned char* prow = smem + U::kP + (s & 1) * U::kPBytes + (row >> 3) * 1024 + (row & 7) * 16 + half * 4 * 128;
#pragma unroll
    for (int c = 0; c < KH / 8; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p0 = ex2(sv[c * 8 + 2 * e] - mnew), p1 = ex2(sv[c * 8 + 2 * e + 1] - mnew);
        lrow += p0 + p1;
        w[e] = M::pack(p0, p1);
      }
      *reinterpret_cast<uint4*>(prow + c * 128) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    // the previous stage's P V is folded before this stage's overwrites its accumulator
    if (s > 0 && !(ok = fold(s - 1))) break;
    alpha_prev = alpha;
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < kUKeys / 16; ++kk)
        umma_f16(t_o, umma_desc(sb + U::kP + (s & 1) * U::kPBytes + kk * 256, 128, 1024),
                 umma_desc(sb + U::kV + (s % kUKV) * U::kKVBytes + kk * 256, 128, U::kVChunk), idesc_o, kk > 0);
      umma_commit(bar_o);
    }
    // stage s + 2 into the buffer of stage s - 1 (its S and P V are done)
    if (s + 2 < n_st) load_kv(s + 2, (s + 2) % kUKV, next_blk);
    cp_async_commit();
    if (s + 3 < n_st) next_blk = table_entry(s + 3);
  }
  if (ok) ok = fold(n_st - 1);
  cp_async_wait<0>();
  if (!ok && tid == 0) record_status(a.status, AUGUR_KV_ETIMEOUT);
  red_l[half * kURows + row] = lrow;  // both halves' sums share one maximum per stage
  __syncthreads();
  lrow = red_l[row] + red_l[kURows + row];
  if (ok && slot < a.groups && i0 + tok < n) {
    const float inv = lrow > 0.f ? 1.f / lrow : 0.f;
    char* orow = a.out + int64_t(q0 + i0 + tok) * a.out_stride_t + int64_t(hk * a.groups + slot) * a.out_stride_h +
                 half * DH * 2;
#pragma unroll
    for (int c = 0; c < DH / 8; ++c) {
      uint4 w;
      w.x = M::pack(o[c * 8 + 0] * inv, o[c * 8 + 1] * inv);
      w.y = M::pack(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv);
      w.z = M::pack(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv);
      w.w = M::pack(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv);
      *reinterpret_cast<uint4*>(orow + c * 16) = w;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(U::kCols) : "memory");
}

template <typename T, int D>
int launch_umma(const PrefillArgs& a, cudaStream_t st) {
  using augur_kv_dev::fail;
  constexpr int smem = UCfg<D>::kBytes;
  static int attr_done[augur_kv_dev::kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= augur_kv_dev::kMaxDevices)
    return fail(AUGUR_KV_ECUDA, "paged_prefill_attention: cannot query the current device");
  {
    std::lock_guard<std::recursive_mutex> lock(augur_kv_dev::g_cache_mutex);
    if (!attr_done[dev]) {
      if (cudaFuncSetAttribute(attn_prefill_umma_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
          cudaSuccess)
        return augur_kv_dev::check_launch("cudaFuncSetAttribute(attn_prefill_umma_kernel)");
      attr_done[dev] = 1;
    }
  }
  const dim3 grid{unsigned((a.max_q_len + kQT - 1) / kQT), unsigned(a.batch * a.hkv), 1u};
  attn_prefill_umma_kernel<T, D><<<grid, unsigned(kUThreads), smem, st>>>(a);
  return augur_kv_dev::check_launch("attn_prefill_umma_kernel");
}

// ---------------------------------------------------------------------------
// Generic path: one CTA per (query token, query head), the reference's order
// ---------------------------------------------------------------------------

constexpr int kGenericThreads = 128;

__device__ __forceinline__ float load_elem(const char* p, int dtype) {
  if (dtype == AUGUR_KV_F32) return *reinterpret_cast<const float*>(p);
  if (dtype == AUGUR_KV_F16) return __half2float(*reinterpret_cast<const __half*>(p));
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
}
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

__global__ void __launch_bounds__(kGenericThreads) attn_prefill_generic_kernel(PrefillArgs a) {
  extern __shared__ __align__(16) float gsm[];
  const int D = a.head_dim;
  float* qv = gsm;                    // head_dim
  float* red = qv + D;                // kGenericThreads
  float* sc = red + kGenericThreads;  // scores of keys [0, position]
  const int hq = blockIdx.x, i = blockIdx.y, b = blockIdx.z;
  int q0, n, past;
  if (!seq_bounds(a, b, q0, n, past)) return;
  if (i >= n) return;
  const int nk = past + i + 1;  // keys [0, position]
  const int hk = hq / a.groups;
  const int es = a.dtype == AUGUR_KV_F32 ? 4 : 2;
  const char* qrow = a.q + int64_t(q0 + i) * a.q_stride_t + int64_t(hq) * a.q_stride_h;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qv[d] = load_elem(qrow + int64_t(d) * es, a.dtype);
  __syncthreads();
  float local_max = kNegInf;
  for (int pos = threadIdx.x; pos < nk; pos += blockDim.x) {
    const char* kr = pool_row(a, a.k, b, hk, pos);
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
  for (int pos = threadIdx.x; pos < nk; pos += blockDim.x) {
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
  for (int pos = threadIdx.x; pos < nk; pos += blockDim.x) sc[pos] = L > 0.f ? round_to(sc[pos] / L, a.dtype) : 0.f;
  __syncthreads();
  char* orow = a.out + int64_t(q0 + i) * a.out_stride_t + int64_t(hq) * a.out_stride_h;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int pos = 0; pos < nk; ++pos) {
      const char* vr = pool_row(a, a.v, b, hk, pos);
      if (vr != nullptr) acc = fmaf(sc[pos], load_elem(vr + int64_t(d) * es, a.dtype), acc);
    }
    store_elem(orow + int64_t(d) * es, a.dtype, acc);
  }
}

template <typename T, int D>
int launch_mma(const PrefillArgs& a, cudaStream_t st) {
  using augur_kv_dev::fail;
  constexpr int smem = PfCfg<D>::kBytes;
  if (smem > 48 * 1024) {
    static int attr_done[augur_kv_dev::kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= augur_kv_dev::kMaxDevices)
      return fail(AUGUR_KV_ECUDA, "paged_prefill_attention: cannot query the current device");
    std::lock_guard<std::recursive_mutex> lock(augur_kv_dev::g_cache_mutex);
    if (!attr_done[dev]) {
      if (cudaFuncSetAttribute(attn_prefill_mma_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
          cudaSuccess)
        return augur_kv_dev::check_launch("cudaFuncSetAttribute(attn_prefill_mma_kernel)");
      attr_done[dev] = 1;
    }
  }
  const dim3 grid{unsigned((a.max_q_len + kQT - 1) / kQT), unsigned(a.batch * a.hkv), 1u};
  attn_prefill_mma_kernel<T, D><<<grid, unsigned(a.groups * 32), smem, st>>>(a);
  return augur_kv_dev::check_launch("attn_prefill_mma_kernel");
}

}  // namespace augur_kv_pf

#define AUGUR_KV_EXPORT extern "C" __attribute__((visibility("default")))

AUGUR_KV_EXPORT int augur_kv_paged_prefill_attention(
    const void* q, const int64_t* q_strides, const void* k_pool, const void* v_pool, const int64_t* pool_strides,
    int64_t num_blocks, int32_t block_size, const int32_t* block_tables, int64_t tables_stride, int64_t max_blocks,
    const int32_t* seq_lens, const int32_t* q_starts, int32_t batch, int32_t max_q_len, int32_t max_seq_len,
    int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, int32_t dtype, void* out, const int64_t* out_strides,
    int32_t flags, int32_t* status, void* stream) {
  using namespace augur_kv_pf;
  using augur_kv_dev::fail;
  augur_kv_dev::g_last_error[0] = '\0';
  const int es = augur_kv_dev::elem_size(dtype);
  if (es == 0) return fail(AUGUR_KV_EINVAL, "paged_prefill_attention: unknown dtype %d", dtype);
  if (batch < 0 || max_q_len < 0 || max_seq_len < 0)
    return fail(AUGUR_KV_EINVAL, "paged_prefill_attention: negative sizes");
  if (batch == 0 || max_q_len == 0) return AUGUR_KV_OK;
  if (q == nullptr || q_strides == nullptr || k_pool == nullptr || v_pool == nullptr || pool_strides == nullptr ||
      block_tables == nullptr || seq_lens == nullptr || q_starts == nullptr || out == nullptr ||
      out_strides == nullptr)
    return fail(AUGUR_KV_EINVAL, "paged_prefill_attention: null pointer argument");
  if (n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks <= 0 || max_blocks <= 0 || max_q_len > max_seq_len || n_q_heads > 65535 ||
      int64_t(batch) * n_kv_heads > 65535 || max_q_len > 65535)
    return fail(AUGUR_KV_EINVAL, "paged_prefill_attention: bad sizes");
  if (flags != AUGUR_KV_ATTN_AUTO && flags != AUGUR_KV_ATTN_GENERIC && flags != AUGUR_KV_ATTN_TCGEN05 &&
      flags != AUGUR_KV_ATTN_MMA_SYNC)
    return fail(AUGUR_KV_EINVAL, "paged_prefill_attention: unknown flags %d", flags);

  PrefillArgs a;
  memset(&a, 0, sizeof(a));
  a.q = static_cast<const char*>(q);
  a.q_stride_t = q_strides[0] * es;
  a.q_stride_h = q_strides[1] * es;
  a.k = static_cast<const char*>(k_pool);
  a.v = static_cast<const char*>(v_pool);
  a.blk_stride = pool_strides[0] * es;
  a.head_stride = pool_strides[1] * es;
  a.row_stride = pool_strides[2] * es;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz(unsigned(block_size)) : -1;
  a.tables = block_tables;
  a.tables_stride = tables_stride;
  a.max_blocks = max_blocks;
  a.seq_lens = seq_lens;
  a.q_starts = q_starts;
  a.batch = batch;
  a.max_q_len = max_q_len;
  a.max_seq = max_seq_len;
  a.hq = n_q_heads;
  a.hkv = n_kv_heads;
  a.groups = n_q_heads / n_kv_heads;
  a.head_dim = head_dim;
  a.dtype = dtype;
  a.sqrt_d = sqrtf(float(head_dim));
  {
    int e = 0;
    a.scale_exact = frexpf(a.sqrt_d, &e) == 0.5f ? 1 : 0;
    a.inv_sqrt_d = 1.0f / a.sqrt_d;
  }
  a.out = static_cast<char*>(out);
  a.out_stride_t = out_strides[0] * es;
  a.out_stride_h = out_strides[1] * es;
  a.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // tensor cores: a 16-bit dtype, head_dim 64 or 128, at most 8 query heads
  // per KV head, 16-byte aligned rows (q and out: 4-byte aligned pairs)
  const uintptr_t align = reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) |
                          uintptr_t(a.blk_stride) | uintptr_t(a.head_stride) | uintptr_t(a.row_stride);
  const uintptr_t align4 = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) |
                           uintptr_t(a.q_stride_t) | uintptr_t(a.q_stride_h) | uintptr_t(a.out_stride_t) |
                           uintptr_t(a.out_stride_h);
  const bool mma_ok = (dtype == AUGUR_KV_BF16 || dtype == AUGUR_KV_F16) && (head_dim == 64 || head_dim == 128) &&
                      a.groups <= kMaxGroups && (align & 15u) == 0 && (align4 & 3u) == 0 &&
                      a.row_stride == int64_t(head_dim) * es;
  // tcgen05: the same shapes with q and out rows 16-byte aligned (AUTO takes
  // it when it can: 805 against 840 us per layer for mma.sync on the config-4
  // suffix prefill)
  const bool umma_ok = mma_ok && (align4 & 15u) == 0;
  if (flags == AUGUR_KV_ATTN_TCGEN05 || (flags == AUGUR_KV_ATTN_AUTO && umma_ok)) {
    if (!umma_ok)
      return fail(AUGUR_KV_EINVAL,
                  "paged_prefill_attention: the tcgen05 kernel needs bf16/fp16, head_dim 64 or 128, <= 8 query "
                  "heads per KV head and 16-byte aligned rows");
    if (dtype == AUGUR_KV_BF16)
      return head_dim == 64 ? launch_umma<__nv_bfloat16, 64>(a, st) : launch_umma<__nv_bfloat16, 128>(a, st);
    return head_dim == 64 ? launch_umma<__half, 64>(a, st) : launch_umma<__half, 128>(a, st);
  }
  if (flags == AUGUR_KV_ATTN_MMA_SYNC && !mma_ok)
    return fail(AUGUR_KV_EINVAL,
                "paged_prefill_attention: the mma.sync kernel needs bf16/fp16, head_dim 64 or 128, <= 8 query "
                "heads per KV head and aligned rows");
  if ((flags == AUGUR_KV_ATTN_AUTO || flags == AUGUR_KV_ATTN_MMA_SYNC) && mma_ok) {
    if (dtype == AUGUR_KV_BF16)
      return head_dim == 64 ? launch_mma<__nv_bfloat16, 64>(a, st) : launch_mma<__nv_bfloat16, 128>(a, st);
    return head_dim == 64 ? launch_mma<__half, 64>(a, st) : launch_mma<__half, 128>(a, st);
  }
  // generic: the query token's scores live in shared memory
  const size_t smem = size_t(head_dim + kGenericThreads + max_seq_len) * sizeof(float);
  if (smem > 200 * 1024)
    return fail(AUGUR_KV_EINVAL, "paged_prefill_attention: the generic path is limited to %d positions",
                int(200 * 1024 / sizeof(float)) - head_dim - kGenericThreads);
  {
    static int attr_bytes[augur_kv_dev::kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= augur_kv_dev::kMaxDevices)
      return fail(AUGUR_KV_ECUDA, "paged_prefill_attention: cannot query the current device");
    std::lock_guard<std::recursive_mutex> lock(augur_kv_dev::g_cache_mutex);
    if (smem > 48 * 1024 && size_t(attr_bytes[dev]) < smem) {
      if (cudaFuncSetAttribute(attn_prefill_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               int(200 * 1024)) != cudaSuccess)
        return augur_kv_dev::check_launch("cudaFuncSetAttribute(attn_prefill_generic_kernel)");
      attr_bytes[dev] = 200 * 1024;
    }
  }
  attn_prefill_generic_kernel<<<dim3(unsigned(n_q_heads), unsigned(max_q_len), unsigned(batch)), kGenericThreads,
                                 smem, st>>>(a);
  return augur_kv_dev::check_launch("attn_prefill_generic_kernel");
}
