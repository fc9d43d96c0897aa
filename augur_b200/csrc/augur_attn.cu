// augur_attn.cu — decode attention that reads the paged KV pool directly.
//
// The reference computes a decode step's attention by gathering the whole
// sequence out of the pool position by position (read_paged_kv,
// augur/paged_kv_cache.py:217-220), repeating each K/V head for the query
// heads of its group and running two eager matmuls around a float32
// softmax (augur/attention.py:72-86). Here one launch covers every sequence
// of the batch for one layer, reading each K/V row of the pool once:
//
//  * attn_decode_mma_kernel (bf16 / fp16, head_dim 64 or 128, <= 16 query
//    heads per KV head): one cluster of up to 8 CTAs per (sequence, KV head)
//    splits the sequence; each warp walks 16-token tiles staged in shared
//    memory with cp.async, computes the group's scores and the P.V product
//    with mma.sync m16n8k16 (the group's query heads are the 16 rows, the
//    tile's tokens the columns), and keeps an online softmax. Warps combine
//    in shared memory, CTAs of the cluster through distributed shared memory
//    into rank 0, which writes the output; no global scratch.
//  * attn_decode_generic_kernel (any dtype / shape): one CTA per (sequence,
//    query head), scores of the whole sequence in shared memory, then the
//    reference's order of operations: max, exp, sum, normalise, P.V.
//
// Rounding follows the reference where it rounds: scores are rounded to the
// cache dtype after q.k and again after the division by sqrt(head_dim)
// (the bf16/fp16 matmul output and the scalar division both produce the
// dtype); probabilities are rounded before the product with V; the output
// is rounded once. Summation order differs, so results agree within a
// floating-point tolerance, not bit for bit.
//
// The decode query sits at the last position of its sequence, so the causal
// mask hides nothing; tokens at or past seq_len are never read.

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "augur_kv.h"
#include "common.cuh"

namespace cg = cooperative_groups;

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
  int32_t max_seq;  // generic kernel: shared-memory score capacity
  int32_t* status;
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

constexpr int kAttnWarps = 4;
constexpr int kTile = 16;  // tokens per tile

template <int D>
struct MmaSmem {
  static constexpr int kStages = 3;             // tiles in flight per warp
  static constexpr int kRowBytes = D * 2 + 16;  // padded: ldmatrix rows hit distinct banks
  static constexpr int kTileBytes = kTile * kRowBytes;
  static constexpr int kPipe = kAttnWarps * kStages * 2 /*K,V*/ * kTileBytes;
  // after the token loop the warps' partial results reuse the pipeline buffers
  static constexpr int kPartO = kAttnWarps * 16 * D * 4;
  static constexpr int kPartML = kAttnWarps * 16 * 4;
  static_assert(kPartO + 2 * kPartML <= kPipe, "partials must fit in the pipeline buffers");
  static constexpr int kCtaO = 16 * D * 4;
  static constexpr int kBytes = kPipe + kCtaO + (2 * 16 + kAttnWarps * 16 + 3 * 8 * 16 + 16) * 4;
};

template <typename T, int D>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_mma_kernel(AttnArgs a) {
  using SM = MmaSmem<D>;
  constexpr int CHUNKS = D * 2 / 16;  // 16-byte pieces per row
  constexpr int DT = MmaType<T>::dtype;
  extern __shared__ __align__(128) unsigned char smem[];
  float* part_o = reinterpret_cast<float*>(smem);  // aliases the pipeline after the loop
  float* part_m = reinterpret_cast<float*>(smem + SM::kPartO);
  float* part_l = part_m + kAttnWarps * 16;
  float* cta_o = reinterpret_cast<float*>(smem + SM::kPipe);
  float* cta_m = cta_o + 16 * D;
  float* cta_l = cta_m + 16;
  float* fac = cta_l + 16;            // [warps][16] rescale factors
  float* rm = fac + kAttnWarps * 16;  // [8 ranks][16] gathered row maxima
  float* rl = rm + 8 * 16;            // [8][16] gathered row sums
  float* rf = rl + 8 * 16;            // [8][16] rescale factors per rank
  float* rL = rf + 8 * 16;            // [16] combined row sums

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = int(cluster.block_rank());
  const int nsplit = int(cluster.num_blocks());
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int G = a.groups;
  const int S = max(0, __ldg(a.seq_lens + b));

  const int tiles = (S + kTile - 1) / kTile;
  const int per_cta = (tiles + nsplit - 1) / nsplit;
  const int tile0 = rank * per_cta;
  const int tile1 = min(tiles, tile0 + per_cta);

  // Query rows of this KV head's group as mma A fragments (rows >= G are 0).
  uint32_t qa[D / 16][4];
  {
    const char* qb = a.q + int64_t(b) * a.q_stride_b;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = g + ((r & 1) ? 8 : 0);
        const int col = ks * 16 + 2 * t + ((r & 2) ? 8 : 0);
        uint32_t v = 0;
        if (row < G) v = *reinterpret_cast<const uint32_t*>(qb + int64_t(hk * G + row) * a.q_stride_h + col * 2);
        qa[ks][r] = v;
      }
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {kNegInf, kNegInf}, lrow[2] = {0.f, 0.f};

  constexpr int NST = SM::kStages;
  unsigned char* wbuf = smem + warp * (NST * 2 * SM::kTileBytes);
  // Each lane copies a fixed 16-byte column (part) of RPL rows of every
  // tile, for K and V alike: one table lookup per row serves both.
  constexpr int RPL = CHUNKS / 2;           // rows per lane per tile
  constexpr int ROW_STEP = 32 / CHUNKS;     // row distance between a lane's rows
  const int part = lane % CHUNKS;
  const int row_base = lane / CHUNKS;
  auto load_tile = [&](int tile, int st) {
    unsigned char* kdst = wbuf + (st * 2 + 0) * SM::kTileBytes + part * 16;
    unsigned char* vdst = wbuf + (st * 2 + 1) * SM::kTileBytes + part * 16;
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      const int r = row_base + i * ROW_STEP;
      const int pos = tile * kTile + r;
      const char* kp = a.k;
      const char* vp = a.v;
      int bytes = 0;
      if (pos < S) {
        const char* rk = row_addr(a, a.k, b, hk, pos);
        if (rk != nullptr) {
          kp = rk + part * 16;
          vp = a.v + (rk - a.k) + part * 16;
          bytes = 16;
        }
      }
      cp_async16(kdst + r * SM::kRowBytes, kp, bytes);
      cp_async16(vdst + r * SM::kRowBytes, vp, bytes);
    }
    cp_async_commit();
  };

  const int my_first = tile0 + warp;
  const int n_my = my_first < tile1 ? (tile1 - my_first + kAttnWarps - 1) / kAttnWarps : 0;
#pragma unroll
  for (int i = 0; i < NST - 1; ++i) {
    if (i < n_my) load_tile(my_first + i * kAttnWarps, i);
    else cp_async_commit();
  }
  for (int it = 0; it < n_my; ++it) {
    const int nxt = it + NST - 1;
    if (nxt < n_my) load_tile(my_first + nxt * kAttnWarps, nxt % NST);
    else cp_async_commit();
    cp_async_wait<NST - 1>();
    __syncwarp();
    const int tile = my_first + it * kAttnWarps;
    const int stage = it % NST;
    const unsigned char* Ks = wbuf + (stage * 2 + 0) * SM::kTileBytes;
    const unsigned char* Vs = wbuf + (stage * 2 + 1) * SM::kTileBytes;

    // scores: 16 query rows x 16 tokens, two n8 tiles
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int mat = lane >> 3, r8 = lane & 7;
      const int tok = (mat >> 1) * 8 + r8;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t bk[4];
        ldmatrix_x4(bk, Ks + tok * SM::kRowBytes + (ks * 16 + (mat & 1) * 8) * 2);
        mma16816<T>(s[0], qa[ks], bk[0], bk[1]);
        mma16816<T>(s[1], qa[ks], bk[2], bk[3]);
      }
    }
    // round as the reference's dtype matmul and scalar division do; mask the tail
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pos = tile * kTile + nt * 8 + 2 * t + (j & 1);
        const float r = round_to(s[nt][j], DT);
        float x = round_to(a.scale_exact ? r * a.inv_sqrt_d : r / a.sqrt_d, DT);
        s[nt][j] = pos < S ? x : kNegInf;
      }
    }
    float mx[2];
    mx[0] = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    mx[1] = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float alpha[2], mnew[2], sum[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mnew[h] = fmaxf(mrow[h], mx[h]);
      alpha[h] = (mrow[h] == kNegInf) ? 0.f : expf(mrow[h] - mnew[h]);
    }
    float p[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int h = j >> 1;
        const float e = (s[nt][j] == kNegInf) ? 0.f : expf(s[nt][j] - mnew[h]);
        p[nt][j] = e;
        sum[h] += e;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
      sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
      lrow[h] = lrow[h] * alpha[h] + sum[h];
      mrow[h] = mnew[h];
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // P (16 rows x 16 tokens) as the A operand of the P.V product
    uint32_t pa[4];
    pa[0] = pack2<T>(p[0][0], p[0][1]);
    pa[1] = pack2<T>(p[0][2], p[0][3]);
    pa[2] = pack2<T>(p[1][0], p[1][1]);
    pa[3] = pack2<T>(p[1][2], p[1][3]);
    {
      const int mat = lane >> 3, r8 = lane & 7;
      const int tok = (mat & 1) * 8 + r8;
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bv[4];
        ldmatrix_x4_trans(bv, Vs + tok * SM::kRowBytes + (dp * 16 + (mat >> 1) * 8) * 2);
        mma16816<T>(o[2 * dp], pa, bv[0], bv[1]);
        mma16816<T>(o[2 * dp + 1], pa, bv[2], bv[3]);
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with the pipeline buffers the partials reuse

  // warps -> CTA
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = g + ((j & 2) ? 8 : 0);
      part_o[(warp * 16 + row) * D + i * 8 + 2 * t + (j & 1)] = o[i][j];
    }
  }
  if (t == 0) {
    part_m[warp * 16 + g] = mrow[0];
    part_m[warp * 16 + g + 8] = mrow[1];
    part_l[warp * 16 + g] = lrow[0];
    part_l[warp * 16 + g + 8] = lrow[1];
  }
  __syncthreads();
  // warps -> CTA: rescale factors once per (warp, row), then the 16 x D sums
  if (int(threadIdx.x) < G) {
    const int row = threadIdx.x;
    float M = kNegInf;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, part_m[w * 16 + row]);
    float L = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float mw = part_m[w * 16 + row];
      const float f = (mw == kNegInf) ? 0.f : expf(mw - M);
      fac[w * 16 + row] = f;
      L += part_l[w * 16 + row] * f;
    }
    cta_m[row] = M;
    cta_l[row] = L;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int row = i / D, d = i - row * D;
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) O += part_o[(w * 16 + row) * D + d] * fac[w * 16 + row];
    cta_o[row * D + d] = O;
  }
  // CTAs of the cluster, through distributed shared memory: every rank reads
  // all ranks' (m, l), then combines and writes its own slice of the outputs
  cluster.sync();
  if (int(threadIdx.x) < G * nsplit) {
    const int row = threadIdx.x % G, r = threadIdx.x / G;
    rm[r * 16 + row] = cluster.map_shared_rank(cta_m, r)[row];
    rl[r * 16 + row] = cluster.map_shared_rank(cta_l, r)[row];
  }
  __syncthreads();
  if (int(threadIdx.x) < G) {
    const int row = threadIdx.x;
    float M = kNegInf;
    for (int r = 0; r < nsplit; ++r) M = fmaxf(M, rm[r * 16 + row]);
    float L = 0.f;
    for (int r = 0; r < nsplit; ++r) {
      const float mr = rm[r * 16 + row];
      const float f = (mr == kNegInf) ? 0.f : expf(mr - M);
      rf[r * 16 + row] = f;
      L += rl[r * 16 + row] * f;
    }
    rL[row] = L;
  }
  __syncthreads();
  {
    const int total = G * D;
    const int chunk = (total + nsplit - 1) / nsplit;
    const int i0 = rank * chunk, i1 = min(total, i0 + chunk);
    char* ob = a.out + int64_t(b) * a.out_stride_b;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
      const int row = i / D, d = i - row * D;
      float O = 0.f;
      for (int r = 0; r < nsplit; ++r) O += cluster.map_shared_rank(cta_o, r)[row * D + d] * rf[r * 16 + row];
      const float L = rL[row];
      store_elem(ob + int64_t(hk * G + row) * a.out_stride_h + d * 2, DT, L > 0.f ? O / L : 0.f);
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until all ranks have read it
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

template <typename T, int D>
int launch_mma(const AttnArgs& a, int nsplit, cudaStream_t st) {
  using SM = MmaSmem<D>;
  auto kern = attn_decode_mma_kernel<T, D>;
  static bool attr_done[kMaxDevices] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(AUGUR_KV_ECUDA, "paged_decode_attention: cannot query the current device");
  {
    std::lock_guard<std::mutex> lock(g_cache_mutex);
    if (!attr_done[dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kBytes) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(attn_decode_mma_kernel)");
      attr_done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(unsigned(nsplit), unsigned(a.hkv), unsigned(a.batch));
  cfg.blockDim = dim3(kAttnWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = SM::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(nsplit);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return fail(AUGUR_KV_ECUDA, "attn_decode_mma_kernel: %s", cudaGetErrorString(e));
  return check_launch("attn_decode_mma_kernel");
}

}  // namespace

AUGUR_KV_EXPORT int augur_kv_paged_decode_attention(
    const void* q, const int64_t* q_strides, const void* k_pool, const void* v_pool, const int64_t* pool_strides,
    int64_t num_blocks, int32_t block_size, const int32_t* block_tables, int64_t tables_stride, int64_t max_blocks,
    const int32_t* seq_lens, int32_t max_seq_len, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
    int32_t head_dim, int32_t dtype, void* out, const int64_t* out_strides, int32_t flags, int32_t* status,
    void* stream) {
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
  if (flags < AUGUR_KV_ATTN_AUTO || flags > AUGUR_KV_ATTN_GENERIC)
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
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The tensor-core path needs a 16-bit dtype, head_dim 64 or 128, at most 16
  // query heads per KV head, and 16-byte aligned rows.
  uintptr_t align = reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) |
                    uintptr_t(a.blk_stride) | uintptr_t(a.head_stride) | uintptr_t(a.row_stride) |
                    reinterpret_cast<uintptr_t>(q) | uintptr_t(a.q_stride_b) | uintptr_t(a.q_stride_h);
  const bool mma_ok = dtype != AUGUR_KV_F32 && (head_dim == 64 || head_dim == 128) && a.groups <= 16 &&
                      (align & 15u) == 0 && a.row_stride == int64_t(head_dim) * es;
  if (flags != AUGUR_KV_ATTN_GENERIC && mma_ok) {
    // split each sequence over a cluster of CTAs: enough CTAs to cover the
    // SMs, at least one 16-token tile per warp, at most 8 (portable clusters)
    const int tiles = (max_seq_len + kTile - 1) / kTile;
    const int64_t units = int64_t(batch) * n_kv_heads;
    int nsplit = int((4 * int64_t(sm_count()) + units - 1) / units);  // about 4 CTAs per SM
    const int by_len = (tiles + kAttnWarps - 1) / kAttnWarps;            // at least one tile per warp
    if (nsplit > by_len) nsplit = by_len;
    if (nsplit > 8) nsplit = 8;
    if (nsplit < 1) nsplit = 1;
    if (dtype == AUGUR_KV_BF16)
      return head_dim == 64 ? launch_mma<__nv_bfloat16, 64>(a, nsplit, st) : launch_mma<__nv_bfloat16, 128>(a, nsplit, st);
    return head_dim == 64 ? launch_mma<__half, 64>(a, nsplit, st) : launch_mma<__half, 128>(a, nsplit, st);
  }

  // generic path: the whole sequence's scores live in shared memory
  const size_t smem = size_t(head_dim + kGenericThreads + max_seq_len) * sizeof(float);
  if (smem > 200 * 1024)
    return fail(AUGUR_KV_EINVAL, "paged_decode_attention: generic path limited to %d positions",
                int(200 * 1024 / sizeof(float)) - head_dim - kGenericThreads);
  a.max_seq = max_seq_len;
  {
    static int attr_bytes[kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return fail(AUGUR_KV_ECUDA, "paged_decode_attention: cannot query the current device");
    std::lock_guard<std::mutex> lock(g_cache_mutex);
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
