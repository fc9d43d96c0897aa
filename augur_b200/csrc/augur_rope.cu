// augur_rope.cu — rotary position embedding fused with the cache write.
//
// The reference rotates q and k with apply_rope (augur/rope.py:12-40) and
// then writes k and v into the cache (write_kv, augur/kv_cache.py:75-112, or
// write_paged_kv, augur/paged_kv_cache.py:167-192; the call site is
// augur/attention.py:53-71). rope_scatter_kernel does both in one pass: each
// thread owns one 16-byte piece of the first half of a row and the matching
// piece of the second half, rotates q rows into q_out and k rows straight
// into their cache slot, and copies v rows.
//
// Arithmetic follows the reference's order and rounding exactly. In the
// cache dtype T:
//   out[d]         = T( T(x[d]       * cos[d]) + T(-x[d + D/2] * sin[d]) )
//   out[d + D/2]   = T( T(x[d + D/2] * cos[d]) + T( x[d]       * sin[d]) )
// Each product and sum is one float32 operation rounded to nearest (no
// fused multiply-add), then rounded to T. These are the three elementwise
// ops of `q * cos + rotate_half(q) * sin`, each producing a T tensor. cos
// and sin come from a caller-provided table, [n_pos][D/2] in T, built from
// the reference's formula (inv_freq = 1 / theta^(2i/D), angle = pos *
// inv_freq, cos/sin in float32, cast to T). With the same table the result
// is bit-exact.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "augur_kv.h"
#include "common.cuh"

namespace augur_kv_dev {

struct RopeArgs {
  const char* src[2];        // K, V
  int64_t src_stride[2][4];  // bytes: layer, row, col, head
  char* dst[2];
  int64_t dst_stride[4];  // bytes: layer, major, row, head
  const int64_t* index;
  int64_t index_stride[2];  // elements: row, col
  int64_t index_row_base;
  int64_t rows_per_major, num_majors, num_slots;
  const int64_t* pos;
  int64_t pos_stride[2];  // elements: row, col
  const char* cos_t;
  const char* sin_t;
  int64_t n_pos;
  const char* q;
  int64_t q_stride[4];  // bytes: layer, row, col, head
  char* q_out;
  int64_t q_out_stride[4];
  int64_t tokens_per_row, n_tokens;
  int32_t hq, hkv, has_v;
  int32_t half;  // head_dim / 2 elements
  int32_t rc;    // rotated pieces per row (half / VEC)
  int32_t cc;    // copied pieces per V row (head_dim / VEC)
  int32_t tasks; // pieces per token per layer: (hq + hkv) * rc + has_v * hkv * cc
  int32_t sh_rc, sh_cc, sh_rpm;  // log2 of rc, cc, rows_per_major when powers of two, else -1
  int32_t* status;
};

template <typename T> struct RopeType;
template <> struct RopeType<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct RopeType<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct RopeType<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// x * y rounded to T, as the reference's T tensor product.
template <typename T>
__device__ __forceinline__ float mul_t(float x, float y) {
  return RopeType<T>::to_f(RopeType<T>::from_f(__fmul_rn(x, y)));
}

template <typename T, int VEC>
struct Piece {
  T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ Piece<T, VEC> load_piece(const char* p) {
  Piece<T, VEC> r;
  if constexpr (sizeof(Piece<T, VEC>) == 16) {
    *reinterpret_cast<uint4*>(&r) = *reinterpret_cast<const uint4*>(p);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) r.v[i] = reinterpret_cast<const T*>(p)[i];
  }
  return r;
}

template <typename T, int VEC>
__device__ __forceinline__ void store_piece(char* p, const Piece<T, VEC>& r) {
  if constexpr (sizeof(Piece<T, VEC>) == 16) {
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(&r);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) reinterpret_cast<T*>(p)[i] = r.v[i];
  }
}

// Destination (major, row) of index value idx for a token of source row `row`
// (same convention as augur_kv_scatter). False: skip (negative) or EBOUNDS.
__device__ __forceinline__ bool rope_slot(const RopeArgs& a, int64_t row, int64_t idx, int64_t& major,
                                          int64_t& off) {
  if (idx < 0) return false;
  if (a.index_row_base > 0) {
    if (idx >= a.rows_per_major || row >= a.num_majors) {
      record_status(a.status, AUGUR_KV_EBOUNDS);
      return false;
    }
    major = row;
    off = idx;
  } else {
    if (idx >= a.num_slots) {
      record_status(a.status, AUGUR_KV_EBOUNDS);
      return false;
    }
    if (a.sh_rpm >= 0) {
      major = idx >> a.sh_rpm;
      off = idx & (a.rows_per_major - 1);
    } else {  // the host keeps num_slots below 2^31 here
      const uint32_t m = uint32_t(idx) / uint32_t(a.rows_per_major);
      major = m;
      off = idx - int64_t(m) * a.rows_per_major;
    }
  }
  return true;
}

// Row and piece of task j among rows of `per_row` pieces (shift when a power of two).
__device__ __forceinline__ void split_task(int j, int per_row, int sh, int& r, int& c) {
  if (sh >= 0) {
    r = j >> sh;
    c = j & (per_row - 1);
  } else {
    r = j / per_row;
    c = j - r * per_row;
  }
}

// Rotation of one 16-byte piece of each half: o1 = x1*c - x2*s, o2 = x2*c + x1*s,
// each product and the sum rounded to T. The packed bf16x2 / f16x2
// instructions round the exact result once; the reference rounds the float32
// result (itself exact for the products) to T. Rounding to float32 first and
// then to T (8 or 11 bits) equals rounding once, because 24 >= 2 x 11 + 2 (double
// rounding is innocuous for +, -, x under that bound), so both give the same bits.
// The explicit .rn keeps the compiler from contracting into a fused multiply-add.
template <typename T, int VEC>
struct Rotate {
  static __device__ __forceinline__ void run(const Piece<T, VEC>& x1, const Piece<T, VEC>& x2,
                                             const Piece<T, VEC>& c, const Piece<T, VEC>& s, Piece<T, VEC>& o1,
                                             Piece<T, VEC>& o2) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float c_ = RopeType<T>::to_f(c.v[e]), s_ = RopeType<T>::to_f(s.v[e]);
      const float a1 = RopeType<T>::to_f(x1.v[e]), a2 = RopeType<T>::to_f(x2.v[e]);
      o1.v[e] = RopeType<T>::from_f(__fsub_rn(mul_t<T>(a1, c_), mul_t<T>(a2, s_)));
      o2.v[e] = RopeType<T>::from_f(__fadd_rn(mul_t<T>(a2, c_), mul_t<T>(a1, s_)));
    }
  }
};

// 16-bit types: the eight elements of a piece as four packed pairs through
// rope_pair (common.cuh), the sequence the fused decode attention uses too.
template <typename T>
struct RotatePacked {
  static __device__ __forceinline__ void run(const Piece<T, 8>& x1, const Piece<T, 8>& x2, const Piece<T, 8>& c,
                                             const Piece<T, 8>& s, Piece<T, 8>& o1, Piece<T, 8>& o2) {
    const uint32_t* cc = reinterpret_cast<const uint32_t*>(&c);
    const uint32_t* ss = reinterpret_cast<const uint32_t*>(&s);
    o1 = x1;
    o2 = x2;
    uint32_t* p = reinterpret_cast<uint32_t*>(&o1);
    uint32_t* q = reinterpret_cast<uint32_t*>(&o2);
#pragma unroll
    for (int e = 0; e < 4; ++e) rope_pair<T>(p[e], q[e], cc[e], ss[e]);
  }
};
template <>
struct Rotate<__nv_bfloat16, 8> : RotatePacked<__nv_bfloat16> {};
template <>
struct Rotate<__half, 8> : RotatePacked<__half> {};

// One thread per piece (VEC elements of each half of a rotated row, or VEC
// elements of a v row; VEC = 16 bytes, or 1 on the unaligned path) of every
// token of layer blockIdx.y; a token's pieces are consecutive threads: q rows,
// then k rows, then v rows. A thread's source loads do not wait for the
// position and slot loads; only the table row and the destination do.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) rope_scatter_kernel(RopeArgs a) {
  const int layer = blockIdx.y;
  const uint32_t tasks = uint32_t(a.tasks);
  const uint32_t total = uint32_t(a.n_tokens) * tasks;  // < 2^31, checked on the host
  const int q_tasks = a.hq * a.rc, rot_tasks = (a.hq + a.hkv) * a.rc;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t t = i / tasks;
    const int j = int(i - t * tasks);
    int64_t row, col;
    if (a.tokens_per_row == a.n_tokens) {
      row = 0;
      col = t;
    } else {
      const uint32_t tr = t / uint32_t(a.tokens_per_row);
      row = tr;
      col = int64_t(t) - int64_t(tr) * a.tokens_per_row;
    }
    if (j < rot_tasks) {
      const bool is_q = j < q_tasks;
      int r, c;
      split_task(is_q ? j : j - q_tasks, a.rc, a.sh_rc, r, c);
      const char* src = is_q ? a.q + layer * a.q_stride[0] + row * a.q_stride[1] + col * a.q_stride[2] +
                                   r * a.q_stride[3]
                             : a.src[0] + layer * a.src_stride[0][0] + row * a.src_stride[0][1] +
                                   col * a.src_stride[0][2] + r * a.src_stride[0][3];
      const int e0 = c * VEC * int(sizeof(T)), e1 = e0 + a.half * int(sizeof(T));
      const Piece<T, VEC> x1 = load_piece<T, VEC>(src + e0), x2 = load_piece<T, VEC>(src + e1);
      const int64_t p = a.pos[row * a.pos_stride[0] + col * a.pos_stride[1]];
      char* dst;
      if (is_q) {
        dst = a.q_out + layer * a.q_out_stride[0] + row * a.q_out_stride[1] + col * a.q_out_stride[2] +
              r * a.q_out_stride[3];
      } else {
        int64_t major, off;
        if (!rope_slot(a, row, a.index[row * a.index_stride[0] + col * a.index_stride[1]], major, off)) continue;
        dst = a.dst[0] + layer * a.dst_stride[0] + major * a.dst_stride[1] + off * a.dst_stride[2] +
              r * a.dst_stride[3];
      }
      if (p < 0 || p >= a.n_pos) {
        record_status(a.status, AUGUR_KV_EBOUNDS);
        continue;
      }
      const int64_t tab = p * a.half * int64_t(sizeof(T)) + e0;
      const Piece<T, VEC> cs = load_piece<T, VEC>(a.cos_t + tab), sn = load_piece<T, VEC>(a.sin_t + tab);
      Piece<T, VEC> o1, o2;
      Rotate<T, VEC>::run(x1, x2, cs, sn, o1, o2);
      store_piece<T, VEC>(dst + e0, o1);
      store_piece<T, VEC>(dst + e1, o2);
    } else {
      int h, c;
      split_task(j - rot_tasks, a.cc, a.sh_cc, h, c);
      const int e = c * VEC * int(sizeof(T));
      const Piece<T, VEC> x = load_piece<T, VEC>(a.src[1] + layer * a.src_stride[1][0] + row * a.src_stride[1][1] +
                                                 col * a.src_stride[1][2] + h * a.src_stride[1][3] + e);
      int64_t major, off;
      if (!rope_slot(a, row, a.index[row * a.index_stride[0] + col * a.index_stride[1]], major, off)) continue;
      store_piece<T, VEC>(a.dst[1] + layer * a.dst_stride[0] + major * a.dst_stride[1] + off * a.dst_stride[2] +
                              h * a.dst_stride[3] + e,
                          x);
    }
  }
}

// Cache hints of the token-grouped kernel: bit 0, evict-first (.cs) stores of
// the K/V cache rows; bit 1, source loads that do not allocate in L1 (every
// source row is read once). Measured per layer on B200, three interleaved runs
// each: none 8.06-8.09 us, stores only 8.07 us, loads only 7.83-7.91 us,
// both 7.58-7.69 us (77.5-78.6 % of the HBM peak).
#ifndef AUGUR_KV_ROPE_HINTS
#define AUGUR_KV_ROPE_HINTS 3
#endif

template <typename T>
__device__ __forceinline__ Piece<T, 8> rope_src16(const char* p) {
#if AUGUR_KV_ROPE_HINTS & 2
  Piece<T, 8> r;
  uint4 u;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
               : "l"(p));
  *reinterpret_cast<uint4*>(&r) = u;
  return r;
#else
  return load_piece<T, 8>(p);
#endif
}
template <typename T>
__device__ __forceinline__ void rope_cache16(char* p, const Piece<T, 8>& v) {
#if AUGUR_KV_ROPE_HINTS & 1
  const uint4 u = *reinterpret_cast<const uint4*>(&v);
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
               : "memory");
#else
  store_piece<T, 8>(p, v);
#endif
}

// Resident 128-thread CTAs per SM the token-grouped kernel is compiled for.
// 7 (at most 72 registers; 48 bytes spill) makes a config-2-sized prefill, 8,192
// tokens x 16 lanes = 1,024 CTAs, one wave of 7 x 148 = 1,036 slots. Measured
// per layer on B200: 8.14-8.18 us with 7, 8.66-8.73 us with 8 (64 registers,
// spills), 8.85-8.91 us with 6 (a partial second wave), 9.45 us for the
// thread-per-piece kernel.
#ifndef AUGUR_KV_ROPE_TOKEN
#define AUGUR_KV_ROPE_TOKEN 1
#endif
#ifndef AUGUR_KV_ROPE_MIN_CTAS
#define AUGUR_KV_ROPE_MIN_CTAS 7
#endif

// Token-grouped form for 16-bit rows whose halves are whole 16-byte pieces
// (head_dim 64: PH = 4 pieces per half; head_dim 128: PH = 8). LT = 4 PH
// lanes serve one token: lane l owns column piece c = l % PH of the rotated
// rows rg, rg + 4, rg + 8, rg + 12 (rg = l / PH; q heads first, then k
// heads), and v piece l of the token. The token's position and slot are
// loaded once per lane (one request per group), every source load of a
// 16-row block goes out before the first rotation, and the cos / sin pieces
// are loaded once per lane for all of its rows. At augur's shape (14 + 2
// rotated rows, 2 v rows, head_dim 64) a lane moves 9 pieces, and a
// config-2-sized prefill (8,192 tokens) is one resident wave with no tail.
// The host uses it for at most 16 rotated rows per token (q heads + k heads);
// more rows, fp32 and rows that are not 16-byte aligned take
// rope_scatter_kernel.
template <typename T, int PH>
__global__ void __launch_bounds__(128, AUGUR_KV_ROPE_MIN_CTAS) rope_token_kernel(RopeArgs a) {
  constexpr int LT = 4 * PH;
  using P = Piece<T, 8>;
  const int layer = blockIdx.y;
  const int l = int(threadIdx.x) % LT;
  const int c = l % PH, rg = l / PH;
  const int R = a.hq + a.hkv;
  const int nv = a.has_v ? a.hkv * a.cc : 0;
  constexpr int kHalfBytes = PH * 16;  // the second half of a row is a fixed offset from the first
  const int e0 = c * 16;
  const uint32_t groups = (gridDim.x * blockDim.x) / LT;
  for (uint32_t t = (blockIdx.x * blockDim.x + threadIdx.x) / LT; t < uint32_t(a.n_tokens); t += groups) {
    int64_t row, col;
    if (a.tokens_per_row == a.n_tokens) {
      row = 0;
      col = t;
    } else {
      const uint32_t tr = t / uint32_t(a.tokens_per_row);
      row = tr;
      col = int64_t(t) - int64_t(tr) * a.tokens_per_row;
    }
    const int64_t p = a.pos[row * a.pos_stride[0] + col * a.pos_stride[1]];
    const int64_t idx = a.index[row * a.index_stride[0] + col * a.index_stride[1]];
    const char* qbase = a.q + layer * a.q_stride[0] + row * a.q_stride[1] + col * a.q_stride[2];
    const char* kbase = a.src[0] + layer * a.src_stride[0][0] + row * a.src_stride[0][1] + col * a.src_stride[0][2];
    auto src_of = [&](int r) -> const char* {
      return r < a.hq ? qbase + r * a.q_stride[3] : kbase + (r - a.hq) * a.src_stride[0][3];
    };
    // the token's v piece l, loaded with the first block of rotated rows
    P xv;
    int vh = 0, vc = 0;
    if (l < nv) {
      vh = l / (2 * PH);  // v rows are 2 PH pieces
      vc = l % (2 * PH);
      xv = rope_src16<T>(a.src[1] + layer * a.src_stride[1][0] + row * a.src_stride[1][1] +
                         col * a.src_stride[1][2] + vh * a.src_stride[1][3] + vc * 16);
    }
    P x1[4], x2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = rg + 4 * j;
      if (r < R) {
        const char* src = src_of(r);
        x1[j] = rope_src16<T>(src + e0);
        x2[j] = rope_src16<T>(src + e0 + kHalfBytes);
      }
    }
    int64_t major = 0, off = 0;
    const bool slot_ok = rope_slot(a, row, idx, major, off);
    const int64_t dofs = layer * a.dst_stride[0] + major * a.dst_stride[1] + off * a.dst_stride[2];
    if (slot_ok && l < nv) rope_cache16<T>(a.dst[1] + dofs + vh * a.dst_stride[3] + vc * 16, xv);
    char* kdst = a.dst[0] + dofs;
    const bool p_ok = p >= 0 && p < a.n_pos;
    if (!p_ok && l == 0) record_status(a.status, AUGUR_KV_EBOUNDS);
    P cs, sn;
    if (p_ok) {
      const int64_t tab = p * a.half * int64_t(sizeof(T)) + e0;
      cs = load_piece<T, 8>(a.cos_t + tab);
      sn = load_piece<T, 8>(a.sin_t + tab);
    }
    char* qdst = a.q_out + layer * a.q_out_stride[0] + row * a.q_out_stride[1] + col * a.q_out_stride[2];
    auto rotate_store = [&](int r, const P& y1, const P& y2) {
      const bool is_q = r < a.hq;  // rotated q is read by the attention that follows; k goes to its cache row
      char* dst;
      if (is_q) dst = qdst + r * a.q_out_stride[3];
      else if (slot_ok) dst = kdst + (r - a.hq) * a.dst_stride[3];
      else return;
      P o1, o2;
      Rotate<T, 8>::run(y1, y2, cs, sn, o1, o2);
      if (is_q) {
        store_piece<T, 8>(dst + e0, o1);
        store_piece<T, 8>(dst + e0 + kHalfBytes, o2);
      } else {
        rope_cache16<T>(dst + e0, o1);
        rope_cache16<T>(dst + e0 + kHalfBytes, o2);
      }
    };
    if (p_ok) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = rg + 4 * j;
        if (r < R) rotate_store(r, x1[j], x2[j]);
      }
    }
    if (slot_ok) {
      char* vdst = a.dst[1] + dofs;
      for (int pv = l + LT; pv < nv; pv += LT) {  // more v pieces than lanes (more KV heads)
        split_task(pv, a.cc, a.sh_cc, vh, vc);
        const P x = load_piece<T, 8>(a.src[1] + layer * a.src_stride[1][0] + row * a.src_stride[1][1] +
                                     col * a.src_stride[1][2] + vh * a.src_stride[1][3] + vc * 16);
        store_piece<T, 8>(vdst + vh * a.dst_stride[3] + vc * 16, x);
      }
    }
  }
}

}  // namespace augur_kv_dev

using namespace augur_kv_dev;

#define AUGUR_KV_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

int pow2_log(int64_t v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return s;
}

template <typename T, int VEC>
int launch_rope(RopeArgs a, int n_layers, cudaStream_t st) {
  a.rc = a.half / VEC;
  a.cc = 2 * a.half / VEC;
  a.sh_rc = pow2_log(a.rc);
  a.sh_cc = pow2_log(a.cc);
  a.tasks = (a.hq + a.hkv) * a.rc + a.has_v * a.hkv * a.cc;
  const uint64_t total = uint64_t(a.n_tokens) * uint64_t(a.tasks);
  if (total > 0x7FFFFFFFull) return fail(AUGUR_KV_EINVAL, "rope_scatter: more than 2^31 - 1 pieces per layer");
  uint64_t blocks = (total + 255) / 256;
  const uint64_t cap = uint64_t(sm_count()) * 32;
  if (blocks > cap) blocks = cap;
  // At most two waves of resident CTAs; threads loop over the remaining
  // pieces, so no partial last wave leaves SMs idle (measured: 9.3 µs per
  // layer for config-2-sized prefill against 9.6 µs with one CTA per 256
  // pieces).
  const uint64_t waves =
      uint64_t(sm_count()) * uint64_t(resident_ctas(reinterpret_cast<const void*>(rope_scatter_kernel<T, VEC>), 256)) * 2;
  if (blocks > waves) blocks = waves;
  if (blocks < 1) blocks = 1;
  rope_scatter_kernel<T, VEC><<<dim3(unsigned(blocks), unsigned(n_layers)), 256, 0, st>>>(a);
  return check_launch("rope_scatter_kernel");
}

// The token-grouped kernel: lanes of a token = 4 x pieces per half; one
// resident wave of CTAs at most, groups loop over the remaining tokens.
template <typename T, int PH>
int launch_rope_token(RopeArgs a, int n_layers, cudaStream_t st) {
  a.rc = PH;
  a.cc = 2 * PH;
  a.sh_rc = pow2_log(a.rc);
  a.sh_cc = pow2_log(a.cc);
  a.tasks = 0;
  constexpr uint64_t kThreads = 128;
  const uint64_t lanes = uint64_t(a.n_tokens) * 4 * PH;
  uint64_t blocks = (lanes + kThreads - 1) / kThreads;
  const uint64_t wave =
      uint64_t(sm_count()) * uint64_t(resident_ctas(reinterpret_cast<const void*>(rope_token_kernel<T, PH>), kThreads));
  if (blocks > wave) blocks = wave;
  if (blocks < 1) blocks = 1;
  rope_token_kernel<T, PH><<<dim3(unsigned(blocks), unsigned(n_layers)), unsigned(kThreads), 0, st>>>(a);
  return check_launch("rope_token_kernel");
}

template <typename T>
int launch_rope_t(const RopeArgs& a, int n_layers, bool vec, cudaStream_t st) {
  constexpr int V = 16 / int(sizeof(T));
  if constexpr (sizeof(T) == 2) {
    const int half_bytes = a.half * 2;
    const bool token_ok = vec && a.hq + a.hkv <= 16 && AUGUR_KV_ROPE_TOKEN;
    if (token_ok && half_bytes == 64) return launch_rope_token<T, 4>(a, n_layers, st);
    if (token_ok && half_bytes == 128) return launch_rope_token<T, 8>(a, n_layers, st);
  }
  return vec ? launch_rope<T, V>(a, n_layers, st) : launch_rope<T, 1>(a, n_layers, st);
}

}  // namespace

AUGUR_KV_EXPORT int augur_kv_rope_scatter(
    const void* src_k, const void* src_v, const int64_t* src_k_strides, const int64_t* src_v_strides,
    int64_t tokens_per_row, int32_t dtype, void* dst_k, void* dst_v, const int64_t* dst_strides,
    int64_t rows_per_major, int64_t num_majors, const int64_t* index, const int64_t* index_strides,
    int64_t index_row_base, const int64_t* positions, const int64_t* position_strides, const void* rope_cos,
    const void* rope_sin, int64_t rope_positions, const void* q, const int64_t* q_strides, void* q_out,
    const int64_t* q_out_strides, int32_t n_q_heads, int64_t n_tokens, int32_t n_layers, int32_t n_heads,
    int32_t head_dim, int32_t* status, void* stream) {
  g_last_error[0] = '\0';
  const int es = elem_size(dtype);
  if (es == 0) return fail(AUGUR_KV_EINVAL, "rope_scatter: unknown dtype %d", dtype);
  if (n_tokens < 0 || n_layers < 0 || n_q_heads < 0) return fail(AUGUR_KV_EINVAL, "rope_scatter: negative sizes");
  if (n_tokens == 0 || n_layers == 0) return AUGUR_KV_OK;  // empty tensors may have NULL data
  if (src_k == nullptr || dst_k == nullptr || index == nullptr || src_k_strides == nullptr ||
      dst_strides == nullptr || index_strides == nullptr || positions == nullptr || position_strides == nullptr ||
      rope_cos == nullptr || rope_sin == nullptr)
    return fail(AUGUR_KV_EINVAL, "rope_scatter: null pointer argument");
  if ((src_v == nullptr) != (dst_v == nullptr) || (src_v != nullptr && src_v_strides == nullptr))
    return fail(AUGUR_KV_EINVAL, "rope_scatter: src_v, src_v_strides and dst_v go together");
  if (n_q_heads > 0 && (q == nullptr || q_out == nullptr || q_strides == nullptr || q_out_strides == nullptr))
    return fail(AUGUR_KV_EINVAL, "rope_scatter: q, q_out and their strides are needed with n_q_heads > 0");
  if (n_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0 || rows_per_major <= 0 || num_majors < 0 ||
      tokens_per_row <= 0 || rope_positions <= 0)
    return fail(AUGUR_KV_EINVAL, "rope_scatter: bad sizes (head_dim must be even)");
  if (index_row_base != 0 && index_row_base != rows_per_major)
    return fail(AUGUR_KV_EINVAL, "rope_scatter: index_row_base must be 0 or rows_per_major");
  if (n_layers > 65535) return fail(AUGUR_KV_EINVAL, "rope_scatter: more than 65535 layers");
  if (tokens_per_row > n_tokens) tokens_per_row = n_tokens;
  if (n_tokens % tokens_per_row != 0)
    return fail(AUGUR_KV_EINVAL, "rope_scatter: n_tokens must be a multiple of tokens_per_row");
  if (n_tokens > 0x7FFFFFFF) return fail(AUGUR_KV_EINVAL, "rope_scatter: more than 2^31 - 1 tokens");

  RopeArgs a;
  memset(&a, 0, sizeof(a));
  a.has_v = src_v != nullptr ? 1 : 0;
  a.src[0] = static_cast<const char*>(src_k);
  a.src[1] = static_cast<const char*>(a.has_v ? src_v : src_k);
  a.dst[0] = static_cast<char*>(dst_k);
  a.dst[1] = static_cast<char*>(a.has_v ? dst_v : dst_k);
  for (int i = 0; i < 4; ++i) {
    a.src_stride[0][i] = src_k_strides[i] * es;
    a.src_stride[1][i] = (a.has_v ? src_v_strides[i] : src_k_strides[i]) * es;
    a.dst_stride[i] = dst_strides[i] * es;
    a.q_stride[i] = n_q_heads > 0 ? q_strides[i] * es : 0;
    a.q_out_stride[i] = n_q_heads > 0 ? q_out_strides[i] * es : 0;
  }
  a.index = index;
  a.index_stride[0] = index_strides[0];
  a.index_stride[1] = index_strides[1];
  a.index_row_base = index_row_base;
  a.rows_per_major = rows_per_major;
  a.num_majors = num_majors;
  a.num_slots = rows_per_major * num_majors;
  a.sh_rpm = pow2_log(rows_per_major);
  if (a.sh_rpm < 0 && index_row_base == 0 && a.num_slots > 0x7FFFFFFF)
    return fail(AUGUR_KV_EINVAL, "rope_scatter: more than 2^31 slots need a power-of-two block size");
  a.pos = positions;
  a.pos_stride[0] = position_strides[0];
  a.pos_stride[1] = position_strides[1];
  a.cos_t = static_cast<const char*>(rope_cos);
  a.sin_t = static_cast<const char*>(rope_sin);
  a.n_pos = rope_positions;
  a.q = static_cast<const char*>(q);
  a.q_out = static_cast<char*>(q_out);
  a.tokens_per_row = tokens_per_row;
  a.n_tokens = n_tokens;
  a.hq = n_q_heads;
  a.hkv = n_heads;
  a.half = head_dim / 2;
  a.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // 16-byte pieces when both halves of every row and every table row start
  // on 16-byte boundaries; element by element otherwise.
  uintptr_t bits = uintptr_t(int64_t(a.half) * es) | reinterpret_cast<uintptr_t>(src_k) |
                   reinterpret_cast<uintptr_t>(dst_k) | reinterpret_cast<uintptr_t>(rope_cos) |
                   reinterpret_cast<uintptr_t>(rope_sin);
  if (a.has_v) bits |= reinterpret_cast<uintptr_t>(src_v) | reinterpret_cast<uintptr_t>(dst_v);
  if (n_q_heads > 0) bits |= reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(q_out);
  for (int i = 0; i < 4; ++i) {
    bits |= uintptr_t(a.src_stride[0][i]) | uintptr_t(a.src_stride[1][i]) | uintptr_t(a.dst_stride[i]) |
            uintptr_t(a.q_stride[i]) | uintptr_t(a.q_out_stride[i]);
  }
  const bool vec = (bits & 15u) == 0;
  if (dtype == AUGUR_KV_F32) return launch_rope_t<float>(a, n_layers, vec, st);
  if (dtype == AUGUR_KV_F16) return launch_rope_t<__half>(a, n_layers, vec, st);
  return launch_rope_t<__nv_bfloat16>(a, n_layers, vec, st);
}
