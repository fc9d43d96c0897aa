/*
 * kv_oracle.c — CPU restatement of augur's KV-cache data movement.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA path is compared
 * against (tests/, __graft_entry__.smoke(), and bench.py's CPU-baseline leg).
 * Nothing in augur_b200/ links, loads or calls it.
 *
 * Each function restates one loop of the reference (semioz/augur, pure
 * Python/torch), citing the file:line it follows. All are plain row copies:
 * a "row" is head_dim elements of one (layer, token, head) of K or V, and the
 * reference moves rows with torch indexing assignment, which for equal dtypes
 * copies the bytes and for different dtypes converts element by element with
 * round-to-nearest-even (Tensor.copy_ semantics). Strides are in elements of
 * the tensor they describe; head_dim elements are contiguous.
 *
 * Threads: functions taking n_threads split independent tokens / runs over
 * POSIX threads; with distinct destination slots (every reference case) the
 * result does not depend on the thread count. Use 1 thread when duplicate
 * slots must resolve "last write wins" as the reference's sequential loop does.
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

#define OR_F32 0
#define OR_F16 1
#define OR_BF16 2

static int esize(int dtype) { return dtype == OR_F32 ? 4 : 2; }

/* bf16 bits -> float: the bf16 bits are the high half of the fp32 bits. */
static float bf16_to_float(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* float -> bf16 with round-to-nearest-even: add 0x7FFF plus the lowest kept
 * bit and truncate; NaN maps to the quiet NaN 0x7FC0. */
static uint16_t float_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0) return 0x7FC0;
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

static float load_f(const char* p, int dtype) {
  if (dtype == OR_F32) {
    float f;
    memcpy(&f, p, 4);
    return f;
  }
  if (dtype == OR_F16) {
    _Float16 h;
    memcpy(&h, p, 2);
    return (float)h;
  }
  uint16_t b;
  memcpy(&b, p, 2);
  return bf16_to_float(b);
}

static void store_f(char* p, int dtype, float f) {
  if (dtype == OR_F32) {
    memcpy(p, &f, 4);
  } else if (dtype == OR_F16) {
    _Float16 h = (_Float16)f; /* IEEE round-to-nearest-even */
    memcpy(p, &h, 2);
  } else {
    uint16_t b = float_to_bf16(f);
    memcpy(p, &b, 2);
  }
}

/* One row assignment `dst[...] = src[...]` of head_dim elements. */
static void copy_row(char* dst, int dst_dtype, const char* src, int src_dtype, int64_t head_dim) {
  if (dst_dtype == src_dtype) {
    memcpy(dst, src, (size_t)head_dim * esize(dst_dtype));
    return;
  }
  const int es = esize(src_dtype), ed = esize(dst_dtype);
  for (int64_t e = 0; e < head_dim; ++e) store_f(dst + e * ed, dst_dtype, load_f(src + e * es, src_dtype));
}

/*
 * write_kv data movement — augur/kv_cache.py:103-106:
 *   for b in range(batch): cache[layer, b, :, positions[b], :] = key[b]
 * key [batch, heads, seq, head_dim] (kstr), cache [layers, batch, heads,
 * max_seq, head_dim] (cstr), positions [batch, seq] (pstr). Positions are
 * assumed validated (kv_cache.py:96-101 raises before any write).
 */
void oracle_write_kv(const void* key, const int64_t* kstr, int src_dtype, void* cache,
                     const int64_t* cstr, int dst_dtype, int64_t layer, const int64_t* positions,
                     const int64_t* pstr, int64_t batch, int64_t heads, int64_t seq,
                     int64_t head_dim) {
  const int es = esize(src_dtype), ed = esize(dst_dtype);
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t s = 0; s < seq; ++s) {
      const int64_t pos = positions[b * pstr[0] + s * pstr[1]];
      for (int64_t h = 0; h < heads; ++h) {
        const char* src = (const char*)key + (b * kstr[0] + h * kstr[1] + s * kstr[2]) * es;
        char* dst = (char*)cache + (layer * cstr[0] + b * cstr[1] + h * cstr[2] + pos * cstr[3]) * ed;
        copy_row(dst, dst_dtype, src, src_dtype, head_dim);
      }
    }
}

/*
 * write_paged_kv data movement for tokens whose (block, offset) the host
 * already resolved — augur/paged_kv_cache.py:188-192:
 *   cache.keys[layer, block, :, offset, :] = key[0, :, t, :]
 * key [1, heads, seq, head_dim] (kstr), pool [layers, blocks, heads,
 * block_size, head_dim] (pstr). blocks[t] / offsets[t] for t < n_tokens.
 */
void oracle_write_paged_tokens(const void* key, const int64_t* kstr, int src_dtype, void* pool,
                               const int64_t* pstr, int dst_dtype, int64_t layer,
                               const int64_t* blocks, const int64_t* offsets, int64_t n_tokens,
                               int64_t heads, int64_t head_dim) {
  const int es = esize(src_dtype), ed = esize(dst_dtype);
  for (int64_t t = 0; t < n_tokens; ++t)
    for (int64_t h = 0; h < heads; ++h) {
      const char* src = (const char*)key + (h * kstr[1] + t * kstr[2]) * es;
      char* dst = (char*)pool + (layer * pstr[0] + blocks[t] * pstr[1] + h * pstr[2] + offsets[t] * pstr[3]) * ed;
      copy_row(dst, dst_dtype, src, src_dtype, head_dim);
    }
}

/*
 * read_paged_kv data movement — augur/paged_kv_cache.py:217-220:
 *   for position in range(seq_len):
 *     out[0, :, position, :] = cache[layer, block_ids[position // bs], :, position % bs, :]
 * out [1, heads, seq_len, head_dim] (ostr).
 */
void oracle_read_paged(const void* pool, const int64_t* pstr, int dtype, int64_t layer,
                       const int64_t* block_ids, int64_t block_size, int64_t seq_len, void* out,
                       const int64_t* ostr, int64_t heads, int64_t head_dim) {
  const int e = esize(dtype);
  for (int64_t p = 0; p < seq_len; ++p) {
    const int64_t blk = block_ids[p / block_size], off = p % block_size;
    for (int64_t h = 0; h < heads; ++h) {
      const char* src = (const char*)pool + (layer * pstr[0] + blk * pstr[1] + h * pstr[2] + off * pstr[3]) * e;
      char* dst = (char*)out + (h * ostr[1] + p * ostr[2]) * e;
      memcpy(dst, src, (size_t)head_dim * e);
    }
  }
}

/*
 * copy_prefix_into_cache data movement — augur/prefix_cache.py:66-73:
 *   cache.keys[:, batch_idx, :, :P, :] = entry.keys.to(dtype=cache.dtype)
 * entry [layers, heads, P, head_dim] (estr), cache as in oracle_write_kv.
 */
void oracle_copy_prefix(const void* entry, const int64_t* estr, int src_dtype, void* cache,
                        const int64_t* cstr, int dst_dtype, int64_t batch_idx, int64_t prefix_len,
                        int64_t layers, int64_t heads, int64_t head_dim) {
  const int es = esize(src_dtype), ed = esize(dst_dtype);
  for (int64_t l = 0; l < layers; ++l)
    for (int64_t h = 0; h < heads; ++h)
      for (int64_t p = 0; p < prefix_len; ++p) {
        const char* src = (const char*)entry + (l * estr[0] + h * estr[1] + p * estr[2]) * es;
        char* dst = (char*)cache + (l * cstr[0] + batch_idx * cstr[1] + h * cstr[2] + p * cstr[3]) * ed;
        copy_row(dst, dst_dtype, src, src_dtype, head_dim);
      }
}

/*
 * Slot scatter over many tokens and layers: the composition of
 * write_paged_kv (augur/paged_kv_cache.py:188-192) over every layer of a
 * batch whose (block, offset) pairs were resolved on the host as
 * slot = block * block_size + offset. A negative slot skips the token.
 * src [layers, tokens, heads, head_dim] (sstr: layer, token, head), pool
 * [layers, blocks, heads, block_size, head_dim] (pstr). Same dtype on both
 * sides (elem bytes each). Tokens are split over n_threads threads.
 */
typedef struct {
  const void *src_k, *src_v;
  const int64_t* sstr;
  void *pool_k, *pool_v;
  const int64_t* pstr;
  int64_t elem;
  const int64_t* slots;
  int64_t block_size, layers, heads, head_dim, t0, t1;
} scatter_job;

static void* scatter_range(void* arg) {
  const scatter_job* j = (const scatter_job*)arg;
  const size_t row = (size_t)j->head_dim * (size_t)j->elem;
  for (int64_t t = j->t0; t < j->t1; ++t) {
    const int64_t slot = j->slots[t];
    if (slot < 0) continue;
    const int64_t blk = slot / j->block_size, off = slot % j->block_size;
    for (int64_t l = 0; l < j->layers; ++l)
      for (int64_t h = 0; h < j->heads; ++h) {
        const int64_t so = (l * j->sstr[0] + t * j->sstr[1] + h * j->sstr[2]) * j->elem;
        const int64_t d = (l * j->pstr[0] + blk * j->pstr[1] + h * j->pstr[2] + off * j->pstr[3]) * j->elem;
        memcpy((char*)j->pool_k + d, (const char*)j->src_k + so, row);
        if (j->src_v) memcpy((char*)j->pool_v + d, (const char*)j->src_v + so, row);
      }
  }
  return NULL;
}

#define OR_MAX_THREADS 256

void oracle_scatter_slots(const void* src_k, const void* src_v, const int64_t* sstr, void* pool_k,
                          void* pool_v, const int64_t* pstr, int64_t elem, const int64_t* slots,
                          int64_t block_size, int64_t layers, int64_t tokens, int64_t heads,
                          int64_t head_dim, int n_threads) {
  if (n_threads < 1) n_threads = 1;
  if (n_threads > OR_MAX_THREADS) n_threads = OR_MAX_THREADS;
  if (n_threads > tokens) n_threads = tokens > 0 ? (int)tokens : 1;
  scatter_job jobs[OR_MAX_THREADS];
  pthread_t th[OR_MAX_THREADS];
  for (int i = 0; i < n_threads; ++i) {
    scatter_job j = {src_k, src_v, sstr, pool_k, pool_v, pstr, elem, slots, block_size,
                     layers, heads, head_dim, tokens * i / n_threads, tokens * (i + 1) / n_threads};
    jobs[i] = j;
  }
  for (int i = 1; i < n_threads; ++i) pthread_create(&th[i], NULL, scatter_range, &jobs[i]);
  scatter_range(&jobs[0]);
  for (int i = 1; i < n_threads; ++i) pthread_join(th[i], NULL);
}

/*
 * Runs of rows between two caches, every layer, K and V, every head: the
 * composition the reference expresses as write_paged_kv / read_paged_kv /
 * copy_prefix_into_cache over whole blocks (augur/paged_kv_cache.py:188-192,
 * :217-220; augur/prefix_cache.py:66-73). runs [n_runs][5] = {src_major,
 * src_row, dst_major, dst_row, n_rows}; strides (layer, major, head, row).
 * Same dtype (elem bytes). Runs are split over n_threads threads.
 */
typedef struct {
  const void *src_k, *src_v;
  const int64_t* sstr;
  void *dst_k, *dst_v;
  const int64_t* dstr;
  int64_t elem;
  const int32_t* runs;
  int64_t layers, heads, head_dim, r0, r1;
} runs_job;

static void* runs_range(void* arg) {
  const runs_job* j = (const runs_job*)arg;
  const size_t row = (size_t)j->head_dim * (size_t)j->elem;
  for (int64_t r = j->r0; r < j->r1; ++r) {
    const int32_t* u = j->runs + r * 5;
    for (int64_t l = 0; l < j->layers; ++l)
      for (int64_t h = 0; h < j->heads; ++h)
        for (int64_t i = 0; i < u[4]; ++i) {
          const int64_t so = (l * j->sstr[0] + (int64_t)u[0] * j->sstr[1] + h * j->sstr[2] +
                              ((int64_t)u[1] + i) * j->sstr[3]) * j->elem;
          const int64_t d = (l * j->dstr[0] + (int64_t)u[2] * j->dstr[1] + h * j->dstr[2] +
                             ((int64_t)u[3] + i) * j->dstr[3]) * j->elem;
          memcpy((char*)j->dst_k + d, (const char*)j->src_k + so, row);
          if (j->src_v) memcpy((char*)j->dst_v + d, (const char*)j->src_v + so, row);
        }
  }
  return NULL;
}

void oracle_copy_runs(const void* src_k, const void* src_v, const int64_t* sstr, void* dst_k,
                      void* dst_v, const int64_t* dstr, int64_t elem, const int32_t* runs,
                      int64_t n_runs, int64_t layers, int64_t heads, int64_t head_dim,
                      int n_threads) {
  if (n_threads < 1) n_threads = 1;
  if (n_threads > OR_MAX_THREADS) n_threads = OR_MAX_THREADS;
  if (n_threads > n_runs) n_threads = n_runs > 0 ? (int)n_runs : 1;
  runs_job jobs[OR_MAX_THREADS];
  pthread_t th[OR_MAX_THREADS];
  for (int i = 0; i < n_threads; ++i) {
    runs_job j = {src_k, src_v, sstr, dst_k, dst_v, dstr, elem, runs, layers, heads, head_dim,
                  n_runs * i / n_threads, n_runs * (i + 1) / n_threads};
    jobs[i] = j;
  }
  for (int i = 1; i < n_threads; ++i) pthread_create(&th[i], NULL, runs_range, &jobs[i]);
  runs_range(&jobs[0]);
  for (int i = 1; i < n_threads; ++i) pthread_join(th[i], NULL);
}

int oracle_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  if (n > OR_MAX_THREADS) n = OR_MAX_THREADS;
  return (int)n;
}
