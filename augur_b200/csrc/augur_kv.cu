// augur_kv.cu — sm_100a kernels and the C ABI of libaugur_kv.so.
//
// Two kernel families move every byte of augur's KV caches:
//
//  * scatter   — token-granular: one source token-layer (K and V, all heads)
//                goes to one slot picked by an index (slot mapping or position).
//                Prefill scatter, decode append, contiguous write_kv.
//                Reference: augur/kv_cache.py:103-106, augur/paged_kv_cache.py:188-192.
//  * copy_runs — run-granular: runs of consecutive rows (a whole 16-token block
//                per head is one 2 KiB run in both layouts) between two caches.
//                Gather, prefix copy, contiguous->paged handoff, copy-on-write.
//                Reference: augur/paged_kv_cache.py:217-220, augur/prefix_cache.py:66-73.
//
// Both are pure copies. Same-dtype moves are byte copies with 16-byte vectors
// (8/4/2/1 when the addresses or row sizes do not allow 16), so results are
// bit-identical to the reference's torch indexing. The copy_runs bulk path
// stages each run through shared memory with TMA bulk copies
// (cp.async.bulk global->shared with an mbarrier, then shared->global in a
// bulk group); no multicast form is used anywhere.
//
// Every index that is dereferenced is bounds-checked in the kernel; a bad one
// records AUGUR_KV_EBOUNDS in the caller's status word and the row is skipped.
// The only wait is the bulk pipeline's mbarrier wait, bounded by kWaitLimitNs
// of %globaltimer time; on expiry it records AUGUR_KV_ETIMEOUT and returns.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdarg.h>
#include <stdint.h>

#include <mutex>
#include <stdio.h>
#include <string.h>

#include "augur_kv.h"
#include "common.cuh"

#define AUGUR_KV_VERSION ((0 << 16) | 6)

namespace augur_kv_dev {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(AUGUR_KV_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return AUGUR_KV_OK;
}

int elem_size(int32_t dtype) {
  switch (dtype) {
    case AUGUR_KV_F32: return 4;
    case AUGUR_KV_F16: return 2;
    case AUGUR_KV_BF16: return 2;
    default: return 0;
  }
}

// log2 of v when v is a positive power of two, else -1.
int pow2_shift(int64_t v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return s;
}

// Guards the per-device launch-configuration caches below; entry points are
// otherwise stateless and may be called from several host threads.
std::recursive_mutex g_cache_mutex;

int sm_count() {
  static int cached[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::recursive_mutex> lock(g_cache_mutex);
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// Resident CTAs per SM of `kernel` at `threads` threads (no dynamic shared
// memory), from the occupancy calculator, cached per device and kernel.
int resident_ctas(const void* kernel, int threads) {
  struct Entry {
    const void* k;
    int dev;
    int n;
  };
  static Entry cache[256];
  static int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::recursive_mutex> lock(g_cache_mutex);
  for (int i = 0; i < used; ++i)
    if (cache[i].k == kernel && cache[i].dev == dev) return cache[i].n;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, 0) != cudaSuccess || n < 1) n = 1;
  if (used < 256) cache[used++] = Entry{kernel, dev, n};
  return n;
}

// x extent of a 2-D (runs x planes) grid: enough CTAs of `warps` warps for
// every run of a plane, but no more than `cap` CTAs over all planes (the
// kernels loop over runs with a stride).
unsigned grid_x(uint64_t n_runs, uint64_t warps, uint64_t planes, uint64_t cap) {
  uint64_t x = (n_runs + warps - 1) / warps;
  uint64_t lim = cap / (planes ? planes : 1);
  if (lim < 1) lim = 1;
  if (x > lim) x = lim;
  if (x < 1) x = 1;
  return unsigned(x);
}

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

template <int VEC> struct VecType;
template <> struct VecType<16> { using T = uint4; };
template <> struct VecType<8> { using T = uint2; };
template <> struct VecType<4> { using T = uint32_t; };
template <> struct VecType<2> { using T = uint16_t; };
template <> struct VecType<1> { using T = uint8_t; };

// Streaming load: the source of a cache move is read exactly once.
template <int VEC>
__device__ __forceinline__ typename VecType<VEC>::T load_stream(const char* p) {
  using T = typename VecType<VEC>::T;
  return __ldcs(reinterpret_cast<const T*>(p));
}
template <>
__device__ __forceinline__ uint4 load_stream<16>(const char* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
template <>
__device__ __forceinline__ uint2 load_stream<8>(const char* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
template <>
__device__ __forceinline__ uint32_t load_stream<4>(const char* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
template <>
__device__ __forceinline__ uint16_t load_stream<2>(const char* p) {
  return *reinterpret_cast<const volatile uint16_t*>(p);
}
template <>
__device__ __forceinline__ uint8_t load_stream<1>(const char* p) {
  return *reinterpret_cast<const volatile uint8_t*>(p);
}

template <int VEC>
__device__ __forceinline__ void store_vec(char* p, typename VecType<VEC>::T v) {
  *reinterpret_cast<typename VecType<VEC>::T*>(p) = v;
}

#ifndef AUGUR_KV_STORE_HINT
#define AUGUR_KV_STORE_HINT 1  // 1: cache-streaming (.cs, evict-first) 16-byte stores in the scatter
#endif

template <int VEC>
__device__ __forceinline__ void store_stream(char* p, typename VecType<VEC>::T v) {
  store_vec<VEC>(p, v);
}
template <>
__device__ __forceinline__ void store_stream<16>(char* p, uint4 v) {
#if AUGUR_KV_STORE_HINT == 1
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
#else
  store_vec<16>(p, v);
#endif
}

// Element conversion for mixed-dtype moves: through fp32, round to nearest even.
__device__ __forceinline__ float load_as_float(const char* p, int dtype) {
  if (dtype == AUGUR_KV_F32) return *reinterpret_cast<const float*>(p);
  if (dtype == AUGUR_KV_F16) return __half2float(*reinterpret_cast<const __half*>(p));
  uint32_t bits = uint32_t(*reinterpret_cast<const uint16_t*>(p)) << 16;
  return __uint_as_float(bits);
}

// fp32 -> bf16 by the round-to-nearest-even bias method (add 0x7FFF plus the
// lowest kept bit, truncate); NaN becomes the quiet NaN 0x7FC0. This is the
// rounding torch's CPU BFloat16 conversion performs.
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0) return 0x7FC0;
  uint32_t bias = 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t((u + bias) >> 16);
}

__device__ __forceinline__ void store_from_float(char* p, int dtype, float f) {
  if (dtype == AUGUR_KV_F32) {
    *reinterpret_cast<float*>(p) = f;
  } else if (dtype == AUGUR_KV_F16) {
    *reinterpret_cast<__half*>(p) = __float2half_rn(f);
  } else {
    *reinterpret_cast<uint16_t*>(p) = float_to_bf16_bits(f);
  }
}

// ---------------------------------------------------------------------------
// Scatter
// ---------------------------------------------------------------------------

struct ScatterArgs {
  const char* src[2];
  int64_t src_stride[2][4];  // bytes: layer, row, col, head
  char* dst[2];
  int64_t dst_stride[4];     // bytes: layer, major, row, head
  const int64_t* index;
  int64_t index_stride[2];   // elements: row, col
  int64_t index_row_base;
  int64_t rows_per_major;
  int64_t num_majors;
  int64_t num_slots;
  uint32_t tokens_per_row;
  uint32_t n_tokens;
  int32_t n_heads;
  int32_t n_kv;
  int32_t vpr;        // units (vectors or elements) per row
  int32_t upt;        // units per token-layer = n_kv * n_heads * vpr
  int32_t sh_upt, sh_vpr, sh_heads, sh_rpm;  // shifts, valid when POW2
  int32_t unit_bytes_src;   // VEC (same dtype) or source element size
  int32_t unit_bytes_dst;
  int32_t src_dtype, dst_dtype;
  int32_t* status;
};

// Source (row, col) of token t of this launch.
__device__ __forceinline__ void scatter_rowcol(const ScatterArgs& a, uint32_t t, int64_t& row, int64_t& col) {
  if (a.tokens_per_row == a.n_tokens) {
    row = 0;
    col = t;
  } else {
    const uint32_t r = t / a.tokens_per_row;
    row = r;
    col = t - r * a.tokens_per_row;
  }
}

// Destination (major, row) of index value idx for a token of source row
// `row`. Returns false for a skipped (negative) or out-of-range index;
// out-of-range records EBOUNDS.
__device__ __forceinline__ bool scatter_slot(const ScatterArgs& a, int64_t row, int64_t idx, int64_t& major,
                                             int64_t& off) {
  if (idx < 0) return false;
  if (a.index_row_base > 0) {
    // contiguous cache: the index is a position inside batch row `row`
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
    } else if (a.num_slots <= 0x7FFFFFFF) {
      const uint32_t m = uint32_t(idx) / uint32_t(a.rows_per_major);
      major = m;
      off = idx - int64_t(m) * a.rows_per_major;
    } else {
      major = idx / a.rows_per_major;
      off = idx - major * a.rows_per_major;
    }
  }
  return true;
}

// Resolve token t through the device index array to (source row, source col,
// destination major, destination row).
__device__ __forceinline__ bool scatter_resolve(const ScatterArgs& a, uint32_t t, int64_t& row,
                                                int64_t& col, int64_t& major, int64_t& off) {
  scatter_rowcol(a, t, row, col);
  const int64_t idx = __ldg(a.index + row * a.index_stride[0] + col * a.index_stride[1]);
  return scatter_slot(a, row, idx, major, off);
}

// Same-dtype scatter: each thread moves ITEMS vectors of VEC bytes; a warp
// covers one token-layer (K and V, both heads) for the 2x64 bf16 shape.
template <int VEC, bool POW2, int ITEMS>
__global__ void __launch_bounds__(256) scatter_vec_kernel(ScatterArgs a) {
  using T = typename VecType<VEC>::T;
  const int64_t layer = blockIdx.y;
  const uint32_t total = a.n_tokens * uint32_t(a.upt);
  const uint32_t base = blockIdx.x * (256u * ITEMS) + threadIdx.x;
  T val[ITEMS];
  char* dptr[ITEMS];
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    dptr[k] = nullptr;
    const uint32_t i = base + uint32_t(k) * 256u;
    if (i >= total) continue;
    uint32_t t, j, r, v, kv, h;
    if (POW2) {
      t = i >> a.sh_upt;
      j = i & uint32_t(a.upt - 1);
      r = j >> a.sh_vpr;
      v = j & uint32_t(a.vpr - 1);
      kv = r >> a.sh_heads;
      h = r & uint32_t(a.n_heads - 1);
    } else {
      t = i / uint32_t(a.upt);
      j = i - t * uint32_t(a.upt);
      r = j / uint32_t(a.vpr);
      v = j - r * uint32_t(a.vpr);
      kv = r / uint32_t(a.n_heads);
      h = r - kv * uint32_t(a.n_heads);
    }
    int64_t row, col, major, off;
    if (!scatter_resolve(a, t, row, col, major, off)) continue;
    const int64_t* ss = a.src_stride[kv];
    const char* s = a.src[kv] + layer * ss[0] + row * ss[1] + col * ss[2] + int64_t(h) * ss[3] +
                    int64_t(v) * VEC;
    dptr[k] = a.dst[kv] + layer * a.dst_stride[0] + major * a.dst_stride[1] + off * a.dst_stride[2] +
              int64_t(h) * a.dst_stride[3] + int64_t(v) * VEC;
    val[k] = load_stream<VEC>(s);
  }
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    if (dptr[k] != nullptr) store_vec<VEC>(dptr[k], val[k]);
  }
}

// Same-dtype scatter, fast path for a power-of-two number of vectors per
// token-layer (UPT; 32 at the augur shape: K+V x 2 heads x 8 x 16 B).
// Each lane owns fixed (kv, head, column) slots, computed once; a warp item is
// TPW tokens x LU layers, so the index lookup and slot decomposition happen
// once per token per LU layers and every lane has LU*UPL loads in flight
// before its stores. Items enumerate (layer group, token group) with the
// token group fastest, so neighbouring warps read neighbouring source rows.
#ifndef AUGUR_KV_SCATTER_LU
#define AUGUR_KV_SCATTER_LU 8  // layers per warp item for large launches
#endif
#ifndef AUGUR_KV_SCATTER_WAVES
#define AUGUR_KV_SCATTER_WAVES 2  // grid = resident CTAs x this, warps stride over items
#endif

#ifndef AUGUR_KV_SCATTER_MIN_CTAS
#define AUGUR_KV_SCATTER_MIN_CTAS 1  // __launch_bounds__ minimum resident CTAs per SM
#endif

template <int VEC, int UPT, int LU>
__global__ void __launch_bounds__(256, AUGUR_KV_SCATTER_MIN_CTAS) scatter_rows_kernel(ScatterArgs a, uint32_t n_token_groups,
                                                           uint32_t n_items, int32_t n_layers) {
  using T = typename VecType<VEC>::T;
  constexpr int LANES = UPT < 32 ? UPT : 32;  // lanes per token
  constexpr int TPW = 32 / LANES;             // tokens per warp item
  constexpr int UPL = UPT / LANES;            // vectors per lane per token-layer
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t sub = lane / LANES;
  const uint32_t ul = lane % LANES;

  const char* sb[UPL];
  char* db[UPL];
  int64_t s_layer[UPL], s_row[UPL], s_col[UPL];
#pragma unroll
  for (int i = 0; i < UPL; ++i) {
    const uint32_t j = ul + uint32_t(i) * LANES;
    const uint32_t r = j >> a.sh_vpr;
    const uint32_t v = j & uint32_t(a.vpr - 1);
    const uint32_t kv = r >> a.sh_heads;
    const uint32_t h = r & uint32_t(a.n_heads - 1);
    const int64_t* ss = a.src_stride[kv];
    sb[i] = a.src[kv] + int64_t(h) * ss[3] + int64_t(v) * VEC;
    s_layer[i] = ss[0];
    s_row[i] = ss[1];
    s_col[i] = ss[2];
    db[i] = a.dst[kv] + int64_t(h) * a.dst_stride[3] + int64_t(v) * VEC;
  }
  const int64_t d_layer = a.dst_stride[0], d_major = a.dst_stride[1], d_row = a.dst_stride[2];

  const uint32_t warps = gridDim.x * (blockDim.x >> 5);
  for (uint32_t w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < n_items; w += warps) {
    const uint32_t tg = w % n_token_groups;
    const uint32_t lg = w / n_token_groups;
    const uint32_t t = tg * TPW + sub;
    if (t >= a.n_tokens) continue;
    int64_t row, col, major, off;
    // the source rows depend only on the token: their loads go out together
    // with the slot-index load, and only the stores wait for the slot
    scatter_rowcol(a, t, row, col);
    const int64_t idx = __ldg(a.index + row * a.index_stride[0] + col * a.index_stride[1]);
    const int l0 = int(lg) * LU;
    const int nl = (n_layers - l0) < LU ? (n_layers - l0) : LU;
    T val[LU][UPL];
#pragma unroll
    for (int k = 0; k < LU; ++k) {
      if (k < nl) {
#pragma unroll
        for (int i = 0; i < UPL; ++i)
          val[k][i] = load_stream<VEC>(sb[i] + int64_t(l0 + k) * s_layer[i] + row * s_row[i] + col * s_col[i]);
      }
    }
    if (!scatter_slot(a, row, idx, major, off)) continue;
    const int64_t dbase = major * d_major + off * d_row;
#pragma unroll
    for (int k = 0; k < LU; ++k) {
      if (k < nl) {
#pragma unroll
        for (int i = 0; i < UPL; ++i) store_stream<VEC>(db[i] + int64_t(l0 + k) * d_layer + dbase, val[k][i]);
      }
    }
  }
}

// Small scatters whose index arrives by value in the kernel parameters (the
// host passes up to AUGUR_KV_INLINE_INDEX_MAX index values; a decode-step
// write of one or a few tokens needs no device index buffer or copy). One
// thread per 16-byte (or narrower) unit of a token-layer, layers on
// blockIdx.y.
struct InlineIndex {
  int64_t v[AUGUR_KV_INLINE_INDEX_MAX];
};

template <int VEC>
__global__ void __launch_bounds__(256) scatter_inline_kernel(ScatterArgs a, InlineIndex ix) {
  using T = typename VecType<VEC>::T;
  const int64_t layer = blockIdx.y;
  const uint32_t total = a.n_tokens * uint32_t(a.upt);
  for (uint32_t i = blockIdx.x * 256u + threadIdx.x; i < total; i += gridDim.x * 256u) {
    const uint32_t t = i / uint32_t(a.upt);
    const uint32_t j = i - t * uint32_t(a.upt);
    const uint32_t r = j / uint32_t(a.vpr);
    const uint32_t v = j - r * uint32_t(a.vpr);
    const uint32_t kv = r / uint32_t(a.n_heads);
    const uint32_t h = r - kv * uint32_t(a.n_heads);
    int64_t idx = -1;
#pragma unroll
    for (int q = 0; q < AUGUR_KV_INLINE_INDEX_MAX; ++q)
      if (uint32_t(q) == t) idx = ix.v[q];
    int64_t row, col, major, off;
    scatter_rowcol(a, t, row, col);
    if (!scatter_slot(a, row, idx, major, off)) continue;
    const int64_t* ss = a.src_stride[kv];
    const char* src = a.src[kv] + layer * ss[0] + row * ss[1] + col * ss[2] + int64_t(h) * ss[3] +
                      int64_t(v) * VEC;
    char* dst = a.dst[kv] + layer * a.dst_stride[0] + major * a.dst_stride[1] + off * a.dst_stride[2] +
                int64_t(h) * a.dst_stride[3] + int64_t(v) * VEC;
    store_vec<VEC>(dst, *reinterpret_cast<const T*>(src));
  }
}

// Mixed-dtype scatter: one element per thread, converted through fp32.
__global__ void __launch_bounds__(256) scatter_convert_kernel(ScatterArgs a) {
  const int64_t layer = blockIdx.y;
  const uint32_t total = a.n_tokens * uint32_t(a.upt);
  for (uint32_t i = blockIdx.x * 256u + threadIdx.x; i < total; i += gridDim.x * 256u) {
    const uint32_t t = i / uint32_t(a.upt);
    const uint32_t j = i - t * uint32_t(a.upt);
    const uint32_t r = j / uint32_t(a.vpr);
    const uint32_t e = j - r * uint32_t(a.vpr);
    const uint32_t kv = r / uint32_t(a.n_heads);
    const uint32_t h = r - kv * uint32_t(a.n_heads);
    int64_t row, col, major, off;
    if (!scatter_resolve(a, t, row, col, major, off)) continue;
    const int64_t* ss = a.src_stride[kv];
    const char* s = a.src[kv] + layer * ss[0] + row * ss[1] + col * ss[2] + int64_t(h) * ss[3] +
                    int64_t(e) * a.unit_bytes_src;
    char* d = a.dst[kv] + layer * a.dst_stride[0] + major * a.dst_stride[1] +
              off * a.dst_stride[2] + int64_t(h) * a.dst_stride[3] + int64_t(e) * a.unit_bytes_dst;
    store_from_float(d, a.dst_dtype, load_as_float(s, a.src_dtype));
  }
}

// ---------------------------------------------------------------------------
// Row runs
// ---------------------------------------------------------------------------

struct RunArgs {
  const char* src[2];
  int64_t src_stride[4];  // bytes: layer, major, row, head
  char* dst[2];
  int64_t dst_stride[4];
  int64_t src_majors, src_rpm, dst_majors, dst_rpm;
  const int32_t* runs;
  uint32_t n_runs;
  int32_t max_rows;
  int32_t n_heads;
  int32_t n_kv;
  int32_t vpr;            // units per row (vectors or elements)
  int32_t sh_vpr;         // shift when vpr is a power of two, else -1
  int32_t row_bytes_dst;  // head_dim * dst element size
  int32_t unit_bytes_src, unit_bytes_dst;
  int32_t src_dtype, dst_dtype;
  int32_t stage_bytes;    // bulk path: bytes per pipeline stage
  int32_t stages;         // bulk path: pipeline depth per warp
  int32_t fence_system;   // every thread ends with a system-scope fence (peer destinations)
  int32_t* status;
};

struct RunItem {
  const char* src;
  char* dst;
  int32_t n_rows;
};

// Run `run` of the (layer, kv, head) plane this CTA row works on. Grids are
// 2-D: blockIdx.y enumerates (layer, kv, head) once per CTA, so the per-run
// work is one descriptor read and the bounds checks.
struct Plane {
  int64_t layer;
  uint32_t kv, h;
};

__device__ __forceinline__ Plane plane_of(const RunArgs& a, uint32_t y) {
  Plane p;
  p.h = y % uint32_t(a.n_heads);
  const uint32_t rest = y / uint32_t(a.n_heads);
  p.kv = rest % uint32_t(a.n_kv);
  p.layer = rest / uint32_t(a.n_kv);
  return p;
}

__device__ __forceinline__ bool run_resolve(const RunArgs& a, const Plane& p, uint32_t run, RunItem& it) {
  const int32_t* r = a.runs + int64_t(run) * 5;
  const int64_t sm = __ldg(r + 0), sr = __ldg(r + 1), dm = __ldg(r + 2), dr = __ldg(r + 3);
  const int32_t n = __ldg(r + 4);
  if (n <= 0) return false;
  if (sm < 0 || sm >= a.src_majors || sr < 0 || sr + n > a.src_rpm || dm < 0 ||
      dm >= a.dst_majors || dr < 0 || dr + n > a.dst_rpm || n > a.max_rows) {
    record_status(a.status, AUGUR_KV_EBOUNDS);
    return false;
  }
  it.src = a.src[p.kv] + p.layer * a.src_stride[0] + sm * a.src_stride[1] + sr * a.src_stride[2] +
           int64_t(p.h) * a.src_stride[3];
  it.dst = a.dst[p.kv] + p.layer * a.dst_stride[0] + dm * a.dst_stride[1] + dr * a.dst_stride[2] +
           int64_t(p.h) * a.dst_stride[3];
  it.n_rows = n;
  return true;
}

// Vector path: one warp per run of one plane, VEC-byte vectors, 4 in flight
// per lane. Dense rows (row stride == row bytes on both sides) are one
// contiguous span; other layouts decompose each vector into (row, column).
template <int VEC, bool DENSE>
__global__ void __launch_bounds__(256) copy_runs_vec_kernel(RunArgs a) {
  using T = typename VecType<VEC>::T;
  const uint32_t lane = threadIdx.x & 31u;
  const Plane p = plane_of(a, blockIdx.y);
  const uint32_t warps = gridDim.x * (blockDim.x >> 5);
  for (uint32_t run = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); run < a.n_runs; run += warps) {
    RunItem it;
    if (!run_resolve(a, p, run, it)) continue;
    const uint32_t units = uint32_t(it.n_rows) * uint32_t(a.vpr);
    for (uint32_t q0 = 0; q0 < units; q0 += 128u) {
      T val[4];
      char* dptr[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        dptr[k] = nullptr;
        const uint32_t q = q0 + uint32_t(k) * 32u + lane;
        if (q >= units) continue;
        int64_t so, dof;
        if (DENSE) {
          so = dof = int64_t(q) * VEC;
        } else {
          uint32_t row, v;
          if (a.sh_vpr >= 0) {
            row = q >> a.sh_vpr;
            v = q & uint32_t(a.vpr - 1);
          } else {
            row = q / uint32_t(a.vpr);
            v = q - row * uint32_t(a.vpr);
          }
          so = int64_t(row) * a.src_stride[2] + int64_t(v) * VEC;
          dof = int64_t(row) * a.dst_stride[2] + int64_t(v) * VEC;
        }
        val[k] = load_stream<VEC>(it.src + so);
        dptr[k] = it.dst + dof;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (dptr[k] != nullptr) store_vec<VEC>(dptr[k], val[k]);
      }
    }
  }
  // Peer destinations: make this thread's stores visible system-wide before
  // the kernel counts as complete, so a ready flag written by later work on
  // the stream cannot overtake them.
  if (a.fence_system) __threadfence_system();
}

// Mixed-dtype path: one warp per run of one plane, one element per lane step.
__global__ void __launch_bounds__(256) copy_runs_convert_kernel(RunArgs a) {
  const uint32_t lane = threadIdx.x & 31u;
  const Plane p = plane_of(a, blockIdx.y);
  const uint32_t warps = gridDim.x * (blockDim.x >> 5);
  for (uint32_t run = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); run < a.n_runs; run += warps) {
    RunItem it;
    if (!run_resolve(a, p, run, it)) continue;
    const uint32_t units = uint32_t(it.n_rows) * uint32_t(a.vpr);
    for (uint32_t q = lane; q < units; q += 32u) {
      const uint32_t row = q / uint32_t(a.vpr);
      const uint32_t e = q - row * uint32_t(a.vpr);
      const float f = load_as_float(
          it.src + int64_t(row) * a.src_stride[2] + int64_t(e) * a.unit_bytes_src, a.src_dtype);
      store_from_float(it.dst + int64_t(row) * a.dst_stride[2] + int64_t(e) * a.unit_bytes_dst,
                       a.dst_dtype, f);
    }
  }
  if (a.fence_system) __threadfence_system();
}

// --- TMA bulk path ----------------------------------------------------------

constexpr int kBulkMaxStages = 8;
constexpr int kBulkWarps = 4;
constexpr int kBulkBarBytes = 128 * ((kBulkWarps * kBulkMaxStages * 8 + 127) / 128);
constexpr int kBulkSmemBudget = 200 * 1024;      // per CTA, of the 227 KB limit
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // bound on one mbarrier wait
#ifndef AUGUR_KV_BULK_LAG
#define AUGUR_KV_BULK_LAG 4  // stores allowed in flight behind the one just issued
#endif
constexpr int kBulkLag = AUGUR_KV_BULK_LAG;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, for at most
// kWaitLimitNs of %globaltimer time; false when the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_addr(smem_src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Per-lane window of resolved run geometry: lane i holds item base + i, so a
// warp resolves 32 descriptors with one round of loads and the issuing lane
// reads item c with one shuffle.
struct RunWindow {
  uint32_t base;
  const char* src;
  char* dst;
  uint32_t bytes;  // 0 = nothing to move (skipped or out of range)
};

__device__ __forceinline__ void window_fill(const RunArgs& a, const Plane& p, uint32_t gw, uint32_t tw,
                                            uint32_t n, uint32_t base, uint32_t lane, RunWindow& w) {
  w.base = base;
  w.bytes = 0;
  w.src = nullptr;
  w.dst = nullptr;
  const uint32_t c = base + lane;
  RunItem it;
  if (c < n && run_resolve(a, p, gw + c * tw, it)) {
    w.src = it.src;
    w.dst = it.dst;
    w.bytes = uint32_t(it.n_rows) * uint32_t(a.row_bytes_dst);
  }
}

// Warp-uniform read of item c from the window (refilled when c leaves it).
__device__ __forceinline__ void window_get(const RunArgs& a, const Plane& p, uint32_t gw, uint32_t tw,
                                           uint32_t n, uint32_t c, uint32_t lane, RunWindow& w,
                                           const char*& src, char*& dst, uint32_t& bytes) {
  if (c >= w.base + 32u) window_fill(a, p, gw, tw, n, c & ~31u, lane, w);
  const int from = int(c - w.base);
  src = reinterpret_cast<const char*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(w.src), from));
  dst = reinterpret_cast<char*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(w.dst), from));
  bytes = __shfl_sync(0xffffffffu, w.bytes, from);
}

// Each warp runs an independent pipeline of a.stages shared-memory stages
// over the runs gw, gw + total_warps, ... of its CTA row's (layer, kv, head)
// plane: lane 0 bulk-loads item c into stage c % stages and, once that
// stage's mbarrier phase completes, bulk-stores it out. A stage is refilled
// once the store that last read it has finished reading (wait_group.read 1
// keeps one store in flight behind the one just issued). The other lanes
// resolve run descriptors ahead of lane 0 (two windows: loads run up to
// `stages` items ahead of stores).
__global__ void __launch_bounds__(kBulkWarps * 32) copy_runs_bulk_kernel(RunArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t S = uint32_t(a.stages);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kBulkMaxStages;
  unsigned char* buf = smem + kBulkBarBytes + size_t(warp) * S * size_t(a.stage_bytes);
  const Plane p = plane_of(a, blockIdx.y);
  const uint32_t gw = blockIdx.x * kBulkWarps + warp;
  const uint32_t tw = gridDim.x * kBulkWarps;
  if (gw >= a.n_runs) return;  // warp-uniform
  const uint32_t n = (a.n_runs - gw + tw - 1) / tw;

  if (lane == 0) {
    for (uint32_t s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncwarp();

  RunWindow wl, ws;  // load window, store window
  window_fill(a, p, gw, tw, n, 0, lane, wl);
  ws = wl;

  auto issue_load = [&](uint32_t c) {
    const char* src;
    char* dst;
    uint32_t bytes;
    window_get(a, p, gw, tw, n, c, lane, wl, src, dst, bytes);
    if (lane == 0) {
      const uint32_t s = c % S;
      if (bytes != 0) {
        mbar_arrive_expect_tx(&bars[s], bytes);
        bulk_load(buf + size_t(s) * a.stage_bytes, src, bytes, &bars[s]);
      } else {
        mbar_arrive(&bars[s]);  // completes the phase with nothing to move
      }
    }
  };

  const uint32_t prologue = n < S ? n : S;
  for (uint32_t c = 0; c < prologue; ++c) issue_load(c);

  uint32_t c = 0;
  for (; c < n; ++c) {
    const uint32_t s = c % S;
    uint32_t ok = 1;
    if (lane == 0) ok = mbar_wait(&bars[s], (c / S) & 1u) ? 1u : 0u;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) break;
    const char* src;
    char* dst;
    uint32_t bytes;
    window_get(a, p, gw, tw, n, c, lane, ws, src, dst, bytes);
    if (lane == 0) {
      if (bytes != 0) bulk_store(dst, buf + size_t(s) * a.stage_bytes, bytes);
      bulk_commit();
    }
    // Refill the stage of item c - kBulkLag once its store has finished
    // reading shared memory (all but the kBulkLag newest bulk groups).
    if (c >= uint32_t(kBulkLag) && c - kBulkLag + S < n) {
      if (lane == 0) bulk_wait_read<kBulkLag>();
      issue_load(c - kBulkLag + S);
    }
  }
  if (lane == 0) {
    if (c < n) {
      record_status(a.status, AUGUR_KV_ETIMEOUT);
      // Loads issued so far: items [0, prologue) and the refills c' - lag + S
      // for lag <= c' < c. Wait (bounded) for the ones not yet consumed before
      // this CTA's shared memory can be released.
      uint32_t issued_end = (c <= uint32_t(kBulkLag)) ? prologue : c - kBulkLag + S;
      if (issued_end > n) issued_end = n;
      for (uint32_t d = c + 1; d < issued_end; ++d) mbar_wait(&bars[d % S], (d / S) & 1u);
    }
    bulk_wait_all();
  }
}

}  // namespace augur_kv_dev

using namespace augur_kv_dev;

#define AUGUR_KV_EXPORT extern "C" __attribute__((visibility("default")))

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

AUGUR_KV_EXPORT int augur_kv_version(void) { return AUGUR_KV_VERSION; }

AUGUR_KV_EXPORT const char* augur_kv_last_error(void) { return g_last_error; }

AUGUR_KV_EXPORT int augur_kv_scatter(const void* src_k, const void* src_v, const int64_t* src_k_strides,
                                const int64_t* src_v_strides, int64_t tokens_per_row,
                                int32_t src_dtype, void* dst_k, void* dst_v,
                                const int64_t* dst_strides, int64_t rows_per_major,
                                int64_t num_majors, int32_t dst_dtype, const int64_t* index,
                                const int64_t* index_strides, int64_t index_row_base,
                                int32_t index_on_host, int64_t n_tokens, int32_t n_layers,
                                int32_t n_heads, int32_t head_dim, int32_t* status, void* stream) {
  g_last_error[0] = '\0';
  const int es = elem_size(src_dtype), ed = elem_size(dst_dtype);
  if (es == 0 || ed == 0) return fail(AUGUR_KV_EINVAL, "scatter: unknown dtype %d/%d", src_dtype, dst_dtype);
  if (n_tokens < 0 || n_layers < 0) return fail(AUGUR_KV_EINVAL, "scatter: negative sizes");
  if (n_tokens == 0 || n_layers == 0) return AUGUR_KV_OK;  // empty tensors may have NULL data
  if (src_k == nullptr || dst_k == nullptr || index == nullptr || src_k_strides == nullptr ||
      dst_strides == nullptr || index_strides == nullptr)
    return fail(AUGUR_KV_EINVAL, "scatter: null pointer argument");
  if ((src_v == nullptr) != (dst_v == nullptr))
    return fail(AUGUR_KV_EINVAL, "scatter: src_v and dst_v must both be given or both be NULL");
  if (src_v != nullptr && src_v_strides == nullptr)
    return fail(AUGUR_KV_EINVAL, "scatter: src_v_strides is NULL");
  if (n_tokens < 0 || n_layers < 0 || n_heads <= 0 || head_dim <= 0 || rows_per_major <= 0 ||
      num_majors < 0 || tokens_per_row <= 0)
    return fail(AUGUR_KV_EINVAL, "scatter: bad sizes");
  if (index_row_base != 0 && index_row_base != rows_per_major)
    return fail(AUGUR_KV_EINVAL, "scatter: index_row_base must be 0 or rows_per_major");
  if (n_layers > 65535) return fail(AUGUR_KV_EINVAL, "scatter: more than 65535 layers");
  if (tokens_per_row > n_tokens) tokens_per_row = n_tokens;
  if (n_tokens % tokens_per_row != 0)
    return fail(AUGUR_KV_EINVAL, "scatter: n_tokens must be a multiple of tokens_per_row");
  if (index_on_host != 0 && (n_tokens > AUGUR_KV_INLINE_INDEX_MAX || src_dtype != dst_dtype))
    return fail(AUGUR_KV_EINVAL, "scatter: a host index needs at most %d tokens and equal dtypes",
                AUGUR_KV_INLINE_INDEX_MAX);

  const int n_kv = (src_v != nullptr) ? 2 : 1;
  ScatterArgs a;
  memset(&a, 0, sizeof(a));
  a.src[0] = static_cast<const char*>(src_k);
  a.src[1] = static_cast<const char*>(n_kv == 2 ? src_v : src_k);
  a.dst[0] = static_cast<char*>(dst_k);
  a.dst[1] = static_cast<char*>(n_kv == 2 ? dst_v : dst_k);
  for (int i = 0; i < 4; ++i) {
    a.src_stride[0][i] = src_k_strides[i] * es;
    a.src_stride[1][i] = (n_kv == 2 ? src_v_strides[i] : src_k_strides[i]) * es;
    a.dst_stride[i] = dst_strides[i] * ed;
  }
  a.index = index;
  a.index_stride[0] = index_strides[0];
  a.index_stride[1] = index_strides[1];
  a.index_row_base = index_row_base;
  a.rows_per_major = rows_per_major;
  a.num_majors = num_majors;
  a.num_slots = rows_per_major * num_majors;
  a.tokens_per_row = uint32_t(tokens_per_row);
  a.n_tokens = uint32_t(n_tokens);
  a.n_heads = n_heads;
  a.n_kv = n_kv;
  a.sh_rpm = pow2_shift(rows_per_major);
  a.src_dtype = src_dtype;
  a.dst_dtype = dst_dtype;
  a.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (src_dtype != dst_dtype) {
    a.vpr = head_dim;
    a.upt = n_kv * n_heads * head_dim;
    a.unit_bytes_src = es;
    a.unit_bytes_dst = ed;
    const uint64_t total = uint64_t(n_tokens) * uint64_t(a.upt);
    if (total > 0x7FFFFFFFull) return fail(AUGUR_KV_EINVAL, "scatter: too many elements per layer");
    uint64_t blocks = (total + 255) / 256;
    if (blocks > uint64_t(sm_count()) * 16) blocks = uint64_t(sm_count()) * 16;
    scatter_convert_kernel<<<dim3(unsigned(blocks), unsigned(n_layers)), 256, 0, st>>>(a);
    return check_launch("scatter_convert_kernel");
  }

  // Widest vector that divides the row and every address it will touch.
  const int64_t row_bytes = int64_t(head_dim) * es;
  uintptr_t align_bits = uintptr_t(row_bytes) | reinterpret_cast<uintptr_t>(src_k) |
                         reinterpret_cast<uintptr_t>(dst_k);
  if (n_kv == 2) align_bits |= reinterpret_cast<uintptr_t>(src_v) | reinterpret_cast<uintptr_t>(dst_v);
  for (int i = 0; i < 4; ++i) {
    align_bits |= uintptr_t(a.src_stride[0][i]) | uintptr_t(a.src_stride[1][i]) | uintptr_t(a.dst_stride[i]);
  }
  int vec = 16;
  while (vec > 1 && (align_bits & uintptr_t(vec - 1)) != 0) vec >>= 1;
  a.vpr = int32_t(row_bytes / vec);
  a.upt = n_kv * n_heads * a.vpr;
  const uint64_t total = uint64_t(n_tokens) * uint64_t(a.upt);
  if (total > 0x7FFFFFFFull) return fail(AUGUR_KV_EINVAL, "scatter: too many vectors per layer");

  if (index_on_host != 0) {
    InlineIndex ix;
    for (int q = 0; q < AUGUR_KV_INLINE_INDEX_MAX; ++q) ix.v[q] = -1;
    for (int64_t t = 0; t < n_tokens; ++t) {
      const int64_t row = t / tokens_per_row, col = t % tokens_per_row;
      ix.v[t] = index[row * index_strides[0] + col * index_strides[1]];
    }
    const unsigned blocks = unsigned((total + 255) / 256);
    const dim3 grid{blocks, unsigned(n_layers), 1u};
    switch (vec) {
      case 16: scatter_inline_kernel<16><<<grid, 256, 0, st>>>(a, ix); break;
      case 8: scatter_inline_kernel<8><<<grid, 256, 0, st>>>(a, ix); break;
      case 4: scatter_inline_kernel<4><<<grid, 256, 0, st>>>(a, ix); break;
      case 2: scatter_inline_kernel<2><<<grid, 256, 0, st>>>(a, ix); break;
      default: scatter_inline_kernel<1><<<grid, 256, 0, st>>>(a, ix); break;
    }
    return check_launch("scatter_inline_kernel");
  }
  a.sh_upt = pow2_shift(a.upt);
  a.sh_vpr = pow2_shift(a.vpr);
  a.sh_heads = pow2_shift(n_heads);
  const bool pow2 = a.sh_upt >= 0 && a.sh_vpr >= 0 && a.sh_heads >= 0;

  // Fast path: lane-owned slots, one index lookup per token per layer group.
  if (pow2 && a.upt >= 1 && a.upt <= 128) {
    const int lanes = a.upt < 32 ? a.upt : 32;
    const uint32_t tpw = uint32_t(32 / lanes);
    const uint32_t n_token_groups = uint32_t((n_tokens + tpw - 1) / tpw);
    // Small launches (a decode step: tens of tokens) need every (token, layer)
    // as its own warp item to fill the GPU; large ones group LU layers per
    // item to amortise the index lookup and keep LU loads in flight per lane.
    const uint64_t items1 = uint64_t(n_token_groups) * uint64_t(n_layers);
    const bool grouped = items1 > uint64_t(sm_count()) * 64 * 4;
    constexpr int LU = AUGUR_KV_SCATTER_LU;
    const uint64_t n_items = grouped ? uint64_t(n_token_groups) * uint64_t((n_layers + LU - 1) / LU) : items1;
    if (n_items > 0x7FFFFFFFull) return fail(AUGUR_KV_EINVAL, "scatter: too many tokens");
    // Grid: every resident CTA slot AUGUR_KV_SCATTER_WAVES times, each warp
    // striding over the items, unless there are fewer items than that.
    const uint64_t want = (n_items + 7) / 8;
#define AUGUR_ROWS_LAUNCH_LU(VEC, UPT, LUV)                                                    \
  do {                                                                                         \
    auto kern = scatter_rows_kernel<VEC, UPT, LUV>;                                            \
    uint64_t blocks = uint64_t(sm_count()) * resident_ctas((const void*)kern, 256) *           \
                      AUGUR_KV_SCATTER_WAVES;                                                  \
    if (blocks > want) blocks = want;                                                          \
    kern<<<unsigned(blocks), 256, 0, st>>>(a, n_token_groups, uint32_t(n_items), n_layers);    \
  } while (0)
#define AUGUR_ROWS_LAUNCH(VEC, UPT)                       \
  do {                                                    \
    if (grouped) AUGUR_ROWS_LAUNCH_LU(VEC, UPT, LU);      \
    else AUGUR_ROWS_LAUNCH_LU(VEC, UPT, 1);               \
  } while (0)
#define AUGUR_ROWS_UPT(VEC)                        \
  switch (a.upt) {                                 \
    case 1: AUGUR_ROWS_LAUNCH(VEC, 1); break;      \
    case 2: AUGUR_ROWS_LAUNCH(VEC, 2); break;      \
    case 4: AUGUR_ROWS_LAUNCH(VEC, 4); break;      \
    case 8: AUGUR_ROWS_LAUNCH(VEC, 8); break;      \
    case 16: AUGUR_ROWS_LAUNCH(VEC, 16); break;    \
    case 32: AUGUR_ROWS_LAUNCH(VEC, 32); break;    \
    case 64: AUGUR_ROWS_LAUNCH(VEC, 64); break;    \
    default: AUGUR_ROWS_LAUNCH(VEC, 128); break;   \
  }
    switch (vec) {
      case 16: AUGUR_ROWS_UPT(16); break;
      case 8: AUGUR_ROWS_UPT(8); break;
      case 4: AUGUR_ROWS_UPT(4); break;
      case 2: AUGUR_ROWS_UPT(2); break;
      default: AUGUR_ROWS_UPT(1); break;
    }
#undef AUGUR_ROWS_UPT
#undef AUGUR_ROWS_LAUNCH
#undef AUGUR_ROWS_LAUNCH_LU
    return check_launch("scatter_rows_kernel");
  }
  // Large launches give each thread 4 vectors in flight; small ones (decode
  // append) spread one vector per thread over more CTAs.
  const bool big = total * uint64_t(n_layers) >= uint64_t(sm_count()) * 256 * 16;
  const int items = big ? 4 : 1;
  const uint64_t blocks = (total + 256 * items - 1) / (256 * items);
  const dim3 grid{unsigned(blocks), unsigned(n_layers), 1u};

#define AUGUR_SCATTER_LAUNCH(VEC)                                                        \
  do {                                                                                   \
    if (pow2 && big) scatter_vec_kernel<VEC, true, 4><<<grid, 256, 0, st>>>(a);          \
    else if (pow2) scatter_vec_kernel<VEC, true, 1><<<grid, 256, 0, st>>>(a);            \
    else if (big) scatter_vec_kernel<VEC, false, 4><<<grid, 256, 0, st>>>(a);            \
    else scatter_vec_kernel<VEC, false, 1><<<grid, 256, 0, st>>>(a);                     \
  } while (0)
  switch (vec) {
    case 16: AUGUR_SCATTER_LAUNCH(16); break;
    case 8: AUGUR_SCATTER_LAUNCH(8); break;
    case 4: AUGUR_SCATTER_LAUNCH(4); break;
    case 2: AUGUR_SCATTER_LAUNCH(2); break;
    default: AUGUR_SCATTER_LAUNCH(1); break;
  }
#undef AUGUR_SCATTER_LAUNCH
  return check_launch("scatter_vec_kernel");
}

namespace augur_kv_dev {

// Shared body of augur_kv_copy_runs and augur_kv_copy_runs_noalloc. With
// launch = false it runs every host-side check and returns before the first
// CUDA call, so a caller can reject bad arguments before it touches anything.
int copy_runs_impl(const void* src_k, const void* src_v, const int64_t* src_strides,
                   int64_t src_majors, int64_t src_rows_per_major, int32_t src_dtype,
                   void* dst_k, void* dst_v, const int64_t* dst_strides,
                   int64_t dst_majors, int64_t dst_rows_per_major, int32_t dst_dtype,
                   const int32_t* runs, int64_t n_runs, int32_t max_rows,
                   int32_t n_layers, int32_t n_heads, int32_t head_dim,
                   int32_t flags, int32_t* status, void* stream, bool launch) {
  const int es = elem_size(src_dtype), ed = elem_size(dst_dtype);
  if (es == 0 || ed == 0) return fail(AUGUR_KV_EINVAL, "copy_runs: unknown dtype %d/%d", src_dtype, dst_dtype);
  if (n_runs < 0 || n_layers < 0) return fail(AUGUR_KV_EINVAL, "copy_runs: negative sizes");
  if (n_runs == 0 || n_layers == 0) return AUGUR_KV_OK;  // empty tensors may have NULL data
  if (src_k == nullptr || dst_k == nullptr || runs == nullptr || src_strides == nullptr ||
      dst_strides == nullptr)
    return fail(AUGUR_KV_EINVAL, "copy_runs: null pointer argument");
  if ((src_v == nullptr) != (dst_v == nullptr))
    return fail(AUGUR_KV_EINVAL, "copy_runs: src_v and dst_v must both be given or both be NULL");
  if (n_runs < 0 || n_layers < 0 || n_heads <= 0 || head_dim <= 0 || max_rows <= 0 ||
      src_majors < 0 || dst_majors < 0 || src_rows_per_major < 0 || dst_rows_per_major < 0)
    return fail(AUGUR_KV_EINVAL, "copy_runs: bad sizes");
  if ((flags & ~(3 | AUGUR_KV_COPY_FENCE_SYSTEM)) != 0 || (flags & 3) > AUGUR_KV_COPY_BULK)
    return fail(AUGUR_KV_EINVAL, "copy_runs: unknown flags %d", flags);
  const bool fence_system = (flags & AUGUR_KV_COPY_FENCE_SYSTEM) != 0;
  flags &= 3;
  if (fence_system && flags == AUGUR_KV_COPY_BULK)
    return fail(AUGUR_KV_EINVAL, "copy_runs: the system fence is for the vector path");
  if (fence_system) flags = AUGUR_KV_COPY_VECTOR;
  if (int64_t(max_rows) * head_dim * ed > 16384)
    return fail(AUGUR_KV_EINVAL, "copy_runs: max_rows * row bytes exceeds 16384");
  const int n_kv = (src_v != nullptr) ? 2 : 1;
  const uint64_t planes = uint64_t(n_layers) * uint64_t(n_kv) * uint64_t(n_heads);
  if (planes > 65535) return fail(AUGUR_KV_EINVAL, "copy_runs: more than 65535 (layer, kv, head) planes");
  if (n_runs > 0x7FFFFFFF) return fail(AUGUR_KV_EINVAL, "copy_runs: too many runs");

  RunArgs a;
  memset(&a, 0, sizeof(a));
  a.src[0] = static_cast<const char*>(src_k);
  a.src[1] = static_cast<const char*>(n_kv == 2 ? src_v : src_k);
  a.dst[0] = static_cast<char*>(dst_k);
  a.dst[1] = static_cast<char*>(n_kv == 2 ? dst_v : dst_k);
  for (int i = 0; i < 4; ++i) {
    a.src_stride[i] = src_strides[i] * es;
    a.dst_stride[i] = dst_strides[i] * ed;
  }
  a.src_majors = src_majors;
  a.src_rpm = src_rows_per_major;
  a.dst_majors = dst_majors;
  a.dst_rpm = dst_rows_per_major;
  a.runs = runs;
  a.n_runs = uint32_t(n_runs);
  a.max_rows = max_rows;
  a.n_heads = n_heads;
  a.n_kv = n_kv;
  a.row_bytes_dst = head_dim * ed;
  a.src_dtype = src_dtype;
  a.dst_dtype = dst_dtype;
  a.status = status;
  a.fence_system = fence_system ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = sm_count();

  if (src_dtype != dst_dtype) {
    if (flags == AUGUR_KV_COPY_BULK) return fail(AUGUR_KV_EINVAL, "copy_runs: bulk path needs equal dtypes");
    a.vpr = head_dim;
    a.unit_bytes_src = es;
    a.unit_bytes_dst = ed;
    if (!launch) return AUGUR_KV_OK;
    const dim3 grid{grid_x(uint64_t(n_runs), 8, planes, uint64_t(sms) * 16), unsigned(planes), 1u};
    copy_runs_convert_kernel<<<grid, 256, 0, st>>>(a);
    return check_launch("copy_runs_convert_kernel");
  }

  const int64_t row_bytes = int64_t(head_dim) * es;
  uintptr_t align_bits = uintptr_t(row_bytes) | reinterpret_cast<uintptr_t>(src_k) |
                         reinterpret_cast<uintptr_t>(dst_k);
  if (n_kv == 2) align_bits |= reinterpret_cast<uintptr_t>(src_v) | reinterpret_cast<uintptr_t>(dst_v);
  for (int i = 0; i < 4; ++i) align_bits |= uintptr_t(a.src_stride[i]) | uintptr_t(a.dst_stride[i]);
  const bool dense = a.src_stride[2] == row_bytes && a.dst_stride[2] == row_bytes;
  const bool bulk_ok = dense && (align_bits & 15u) == 0;

  if (flags == AUGUR_KV_COPY_BULK && !bulk_ok)
    return fail(AUGUR_KV_EINVAL, "copy_runs: bulk path needs dense rows and 16-byte alignment");
  // AUTO takes the vector path: on B200 it measured faster than the bulk
  // pipeline for 2 KiB runs (config-3 handoff 6.1 vs 5.4 TB/s).
  if (bulk_ok && flags == AUGUR_KV_COPY_BULK) {
    if (!launch) return AUGUR_KV_OK;
    a.stage_bytes = int32_t(((int64_t(max_rows) * row_bytes + 127) / 128) * 128);
    int stages = (kBulkSmemBudget - kBulkBarBytes) / (kBulkWarps * a.stage_bytes);
    if (stages > kBulkMaxStages) stages = kBulkMaxStages;
    if (stages < kBulkLag + 1) stages = kBulkLag + 1;
    a.stages = stages;
    const int smem = kBulkBarBytes + kBulkWarps * stages * a.stage_bytes;
    static int attr_bytes[kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return fail(AUGUR_KV_ECUDA, "copy_runs: cannot query the current device");
    {
      std::lock_guard<std::recursive_mutex> lock(g_cache_mutex);
      if (smem > 48 * 1024 && attr_bytes[dev] < smem) {
        if (cudaFuncSetAttribute(copy_runs_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess)
          return check_launch("cudaFuncSetAttribute(copy_runs_bulk_kernel)");
        attr_bytes[dev] = smem;
      }
    }
    // One wave: as many CTAs as shared memory allows per SM, spread over the
    // planes; every warp runs its own pipeline over its plane's runs.
    int per_sm = (220 * 1024) / smem;
    if (per_sm < 1) per_sm = 1;
    if (per_sm > 8) per_sm = 8;
    const dim3 grid{grid_x(uint64_t(n_runs), kBulkWarps, planes, uint64_t(sms) * per_sm), unsigned(planes), 1u};
    copy_runs_bulk_kernel<<<grid, kBulkWarps * 32, smem, st>>>(a);
    return check_launch("copy_runs_bulk_kernel");
  }

  if (!launch) return AUGUR_KV_OK;
  int vec = 16;
  while (vec > 1 && (align_bits & uintptr_t(vec - 1)) != 0) vec >>= 1;
  a.vpr = int32_t(row_bytes / vec);
  a.sh_vpr = pow2_shift(a.vpr);
  const dim3 grid{grid_x(uint64_t(n_runs), 8, planes, uint64_t(sms) * 32), unsigned(planes), 1u};
#define AUGUR_RUNS_LAUNCH(VEC)                                                        \
  do {                                                                               \
    if (dense) copy_runs_vec_kernel<VEC, true><<<grid, 256, 0, st>>>(a);              \
    else copy_runs_vec_kernel<VEC, false><<<grid, 256, 0, st>>>(a);                   \
  } while (0)
  switch (vec) {
    case 16: AUGUR_RUNS_LAUNCH(16); break;
    case 8: AUGUR_RUNS_LAUNCH(8); break;
    case 4: AUGUR_RUNS_LAUNCH(4); break;
    case 2: AUGUR_RUNS_LAUNCH(2); break;
    default: AUGUR_RUNS_LAUNCH(1); break;
  }
#undef AUGUR_RUNS_LAUNCH
  return check_launch("copy_runs_vec_kernel");
}

}  // namespace augur_kv_dev

AUGUR_KV_EXPORT int augur_kv_copy_runs(const void* src_k, const void* src_v, const int64_t* src_strides,
                                  int64_t src_majors, int64_t src_rows_per_major, int32_t src_dtype,
                                  void* dst_k, void* dst_v, const int64_t* dst_strides,
                                  int64_t dst_majors, int64_t dst_rows_per_major, int32_t dst_dtype,
                                  const int32_t* runs, int64_t n_runs, int32_t max_rows,
                                  int32_t n_layers, int32_t n_heads, int32_t head_dim,
                                  int32_t flags, int32_t* status, void* stream) {
  g_last_error[0] = '\0';
  return copy_runs_impl(src_k, src_v, src_strides, src_majors, src_rows_per_major, src_dtype, dst_k, dst_v,
                        dst_strides, dst_majors, dst_rows_per_major, dst_dtype, runs, n_runs, max_rows,
                        n_layers, n_heads, head_dim, flags, status, stream, true);
}

// ---------------------------------------------------------------------------
// Peer memory (CUDA IPC) for pushing blocks to another process's GPU
// ---------------------------------------------------------------------------

namespace augur_kv_dev {

// cuMemGetAddressRange through the runtime's driver entry point, so the
// library needs no link-time dependency on libcuda.
typedef int (*MemGetAddressRangeFn)(unsigned long long*, size_t*, unsigned long long);

int allocation_base(const void* ptr, const char** base) {
  static MemGetAddressRangeFn fn = nullptr;
  {
    std::lock_guard<std::recursive_mutex> lock(g_cache_mutex);
    if (fn == nullptr) {
      void* f = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || f == nullptr)
        return fail(AUGUR_KV_ECUDA, "ipc: cuMemGetAddressRange entry point unavailable");
      fn = reinterpret_cast<MemGetAddressRangeFn>(f);
    }
  }
  unsigned long long b = 0;
  size_t size = 0;
  const int rc = fn(&b, &size, reinterpret_cast<unsigned long long>(ptr));
  if (rc != 0 || b == 0) return fail(AUGUR_KV_EINVAL, "ipc: %p is not inside a device allocation (%d)", ptr, rc);
  *base = reinterpret_cast<const char*>(b);
  return AUGUR_KV_OK;
}

}  // namespace augur_kv_dev

AUGUR_KV_EXPORT int augur_kv_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  g_last_error[0] = '\0';
  if (dev_ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(AUGUR_KV_EINVAL, "ipc_export: null pointer argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == AUGUR_KV_IPC_HANDLE_BYTES, "IPC handle size");
  const char* base = nullptr;
  const int rc = allocation_base(dev_ptr, &base);
  if (rc != AUGUR_KV_OK) return rc;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<char*>(base));
  if (e != cudaSuccess) return fail(AUGUR_KV_ECUDA, "ipc_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<const char*>(dev_ptr) - base;
  return AUGUR_KV_OK;
}

AUGUR_KV_EXPORT int augur_kv_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out) {
  g_last_error[0] = '\0';
  if (handle == nullptr || dev_ptr_out == nullptr || offset < 0)
    return fail(AUGUR_KV_EINVAL, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(AUGUR_KV_ECUDA, "ipc_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *dev_ptr_out = static_cast<char*>(base) + offset;
  return AUGUR_KV_OK;
}

AUGUR_KV_EXPORT int augur_kv_ipc_close(void* dev_ptr, int64_t offset) {
  g_last_error[0] = '\0';
  if (dev_ptr == nullptr || offset < 0) return fail(AUGUR_KV_EINVAL, "ipc_close: bad argument");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(dev_ptr) - offset);
  if (e != cudaSuccess) return fail(AUGUR_KV_ECUDA, "ipc_close: cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return AUGUR_KV_OK;
}

// ---------------------------------------------------------------------------
// Ready flags between GPUs (disaggregated handoff)
// ---------------------------------------------------------------------------

namespace augur_kv_dev {

// Release-store `value` to a flag that may live in another GPU's memory.
__global__ void signal_kernel(int32_t* flag, int32_t value) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}

// Spin (acquire loads, with back-off) until *flag >= value or timeout_ns of
// %globaltimer time have passed; on timeout record AUGUR_KV_ETIMEOUT and
// return, so the stream moves on and the context stays usable.
__global__ void wait_kernel(const int32_t* flag, int32_t value, int64_t timeout_ns, int32_t* status) {
  const uint64_t t0 = global_timer_ns();
  uint32_t backoff = 32;
  while (true) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= value) return;
    if (global_timer_ns() - t0 > uint64_t(timeout_ns)) {
      record_status(status, AUGUR_KV_ETIMEOUT);
      return;
    }
    __nanosleep(backoff);
    if (backoff < 4096) backoff <<= 1;
  }
}

}  // namespace augur_kv_dev

constexpr int64_t kMaxWaitNs = 60ll * 1000 * 1000 * 1000;  // cap on any requested wait

AUGUR_KV_EXPORT int augur_kv_signal(int32_t* flag, int32_t value, void* stream) {
  g_last_error[0] = '\0';
  if (flag == nullptr) return fail(AUGUR_KV_EINVAL, "signal: null flag");
  signal_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, value);
  return check_launch("signal_kernel");
}

AUGUR_KV_EXPORT int augur_kv_wait(const int32_t* flag, int32_t value, int64_t timeout_ns, int32_t* status,
                                  void* stream) {
  g_last_error[0] = '\0';
  if (flag == nullptr) return fail(AUGUR_KV_EINVAL, "wait: null flag");
  if (timeout_ns <= 0 || timeout_ns > kMaxWaitNs)
    return fail(AUGUR_KV_EINVAL, "wait: timeout_ns must be in (0, %lld]", (long long)kMaxWaitNs);
  wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, value, timeout_ns, status);
  return check_launch("wait_kernel");
}

// ---------------------------------------------------------------------------
// augur_kv_copy_runs_noalloc: the run copy for callers that cannot allocate
// device memory. The run descriptors, which augur_kv_copy_runs reads from a
// device buffer the caller allocated, are staged instead in this file-scope
// array: AUGUR_KV_NOALLOC_MAX_RUNS x 5 int32 (1.25 MiB), which every GPU that
// loads this library holds until the process exits. All calls share it; a
// call overwrites exactly the n_runs entries its kernel reads, so nothing in
// it needs clearing, and calls whose copies overlap on the GPU (different
// streams) race on it.
// ---------------------------------------------------------------------------

static __device__ __align__(256) int32_t g_noalloc_runs[AUGUR_KV_NOALLOC_MAX_RUNS * 5];

namespace augur_kv_dev {

// Device address of g_noalloc_runs for the current device, looked up once per
// device (the first call on a device) with cudaGetSymbolAddress. Host code
// must never pass &g_noalloc_runs itself: on the host that name is only a
// stand-in for the device symbol.
int noalloc_runs_ptr(int32_t** out) {
  static void* cached[kMaxDevices] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(AUGUR_KV_ECUDA, "copy_runs_noalloc: cannot query the current device");
  std::lock_guard<std::recursive_mutex> lock(g_cache_mutex);
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_runs);
    if (e != cudaSuccess || p == nullptr)
      return fail(AUGUR_KV_ECUDA, "copy_runs_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    cached[dev] = p;
  }
  *out = static_cast<int32_t*>(cached[dev]);
  return AUGUR_KV_OK;
}

}  // namespace augur_kv_dev

AUGUR_KV_EXPORT int augur_kv_copy_runs_noalloc(
    const void* src_k, const void* src_v, const int64_t* src_strides, int64_t src_majors,
    int64_t src_rows_per_major, int32_t src_dtype, void* dst_k, void* dst_v, const int64_t* dst_strides,
    int64_t dst_majors, int64_t dst_rows_per_major, int32_t dst_dtype, const int32_t* host_runs,
    int64_t n_runs, int32_t max_rows, int32_t n_layers, int32_t n_heads, int32_t head_dim, int32_t flags,
    int32_t* status, void* stream) {
  g_last_error[0] = '\0';
  if (n_runs < 0) return fail(AUGUR_KV_EINVAL, "copy_runs_noalloc: negative n_runs");
  if (n_runs > AUGUR_KV_NOALLOC_MAX_RUNS)
    return fail(AUGUR_KV_EINVAL,
                "copy_runs_noalloc: %lld runs exceed the fixed scratch of %d runs; split the call "
                "or use augur_kv_copy_runs with a caller-allocated run buffer",
                (long long)n_runs, AUGUR_KV_NOALLOC_MAX_RUNS);
  if (n_runs == 0 || n_layers == 0) return AUGUR_KV_OK;
  if (host_runs == nullptr) return fail(AUGUR_KV_EINVAL, "copy_runs_noalloc: null host_runs");
  // Every argument check of the copy runs first: a call that is rejected must
  // not overwrite the shared array, which an earlier call on another stream
  // may still be reading.
  int rc = copy_runs_impl(src_k, src_v, src_strides, src_majors, src_rows_per_major, src_dtype, dst_k, dst_v,
                          dst_strides, dst_majors, dst_rows_per_major, dst_dtype, host_runs, n_runs, max_rows,
                          n_layers, n_heads, head_dim, flags, status, stream, false);
  if (rc != AUGUR_KV_OK) return rc;
  int32_t* scratch = nullptr;
  rc = noalloc_runs_ptr(&scratch);
  if (rc != AUGUR_KV_OK) return rc;
  // Stream-ordered staging of the descriptors, then the same launch as
  // augur_kv_copy_runs reading them from the scratch array.
  const cudaError_t e = cudaMemcpyAsync(scratch, host_runs, size_t(n_runs) * 5 * sizeof(int32_t),
                                        cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(AUGUR_KV_ECUDA, "copy_runs_noalloc: staging runs: %s", cudaGetErrorString(e));
  return copy_runs_impl(src_k, src_v, src_strides, src_majors, src_rows_per_major, src_dtype, dst_k, dst_v,
                        dst_strides, dst_majors, dst_rows_per_major, dst_dtype, scratch, n_runs, max_rows,
                        n_layers, n_heads, head_dim, flags, status, stream, true);
}
