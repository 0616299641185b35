// Row-wise memory-bound kernels: PolyNorm (+ fused ·up), RMSNorm (+ residual,
// + embedding gather), GDA post reduction, greedy argmax.
//
// Each is one pass over HBM: one CTA (or one warp) per row, fp32 statistics,
// 16-byte vector loads where the row length allows, results rounded once to
// the storage dtype.
#include <cmath>

#include "common.cuh"

namespace motif {
namespace {

constexpr int kMaxThreads = 1024;

int pick_threads(int64_t vecs_per_row) {
  int t = 32;
  while (t < kMaxThreads && t < vecs_per_row) t <<= 1;
  return t;
}

// Elements per 16-byte vector for T, or 1 when the row or pointers forbid it.
template <typename T>
int vec_width(int64_t dim, std::initializer_list<const void*> ptrs, std::initializer_list<int64_t> strides) {
  constexpr int V = 16 / (int)sizeof(T);
  if (dim % V) return 1;
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) % 16)) return 1;
  for (int64_t s : strides)
    if (s % V) return 1;
  return V;
}

// ---------------------------------------------------------------------------
// PolyNorm: y = w0·x³·rsqrt(mean x⁶+eps) + w1·x²·rsqrt(mean x⁴+eps)
//             + w2·x·rsqrt(mean x²+eps) + b                (mlp.py:13-16)
// With `up`, y = T(polynorm(x)) · up (MotifMLP, model.py:267-268).
// ---------------------------------------------------------------------------
//
// Tensor-parallel split (the intermediate axis sharded over ranks): stats_out receives this
// slice's (Σx², Σx⁴, Σx⁶) per row and nothing else is written; stats_in supplies the sums over
// the whole row (full_dim values, summed across ranks) instead of this slice's.
template <typename T, int V>
__global__ void polynorm_kernel(const T* __restrict__ x, const T* __restrict__ up,
                                int64_t in_stride, const T* __restrict__ w,
                                const T* __restrict__ b, float eps, int dim,
                                T* __restrict__ y, float* __restrict__ stats_out = nullptr,
                                const float* __restrict__ stats_in = nullptr, int full_dim = 0) {
  __shared__ float scratch[32 * 3];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * in_stride;
  float acc[3] = {0.f, 0.f, 0.f};
  if (stats_in) {
    acc[0] = stats_in[row * 3];
    acc[1] = stats_in[row * 3 + 1];
    acc[2] = stats_in[row * 3 + 2];
  } else {
    for (int i = threadIdx.x * V; i < dim; i += blockDim.x * V) {
      float v[V];
      load_vec<T, V>(xr + i, v);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        float v2 = v[j] * v[j];
        float v4 = v2 * v2;
        acc[0] += v2;
        acc[1] += v4;
        acc[2] += v4 * v2;
      }
    }
    block_sum<3>(acc, scratch);
    if (stats_out) {
      if (threadIdx.x == 0) {
        stats_out[row * 3] = acc[0];
        stats_out[row * 3 + 1] = acc[1];
        stats_out[row * 3 + 2] = acc[2];
      }
      return;
    }
  }
  const float inv_d = 1.0f / (float)(stats_in ? full_dim : dim);
  const float rs2 = rsqrtf(acc[0] * inv_d + eps);
  const float rs4 = rsqrtf(acc[1] * inv_d + eps);
  const float rs6 = rsqrtf(acc[2] * inv_d + eps);
  const float w0 = to_f<T>(w[0]), w1 = to_f<T>(w[1]), w2 = to_f<T>(w[2]), bb = to_f<T>(b[0]);
  const T* ur = up ? up + row * in_stride : nullptr;
  T* yr = y + row * (int64_t)dim;
  for (int i = threadIdx.x * V; i < dim; i += blockDim.x * V) {
    float v[V], o[V];
    load_vec<T, V>(xr + i, v);
    float u[V];
    if (ur) load_vec<T, V>(ur + i, u);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float v2 = v[j] * v[j];
      float v3 = v2 * v[j];
      float r = w0 * (v3 * rs6) + w1 * (v2 * rs4) + w2 * (v[j] * rs2) + bb;
      o[j] = ur ? round_through<T>(r) * u[j] : r;
    }
    store_vec<T, V>(yr + i, o);
  }
}

template <typename T>
int launch_polynorm(const void* x, const void* up, int64_t in_stride, const void* w,
                    const void* b, float eps, int64_t rows, int64_t dim, void* y,
                    cudaStream_t st, float* stats_out = nullptr, const float* stats_in = nullptr,
                    int64_t full_dim = 0) {
  const int V = vec_width<T>(dim, {x, up, y}, {in_stride});
  const int threads = pick_threads(ceil_div(dim, V));
  auto xp = static_cast<const T*>(x);
  auto up_p = static_cast<const T*>(up);
  if (V == 1)
    polynorm_kernel<T, 1><<<rows, threads, 0, st>>>(xp, up_p, in_stride, static_cast<const T*>(w),
                                                    static_cast<const T*>(b), eps, (int)dim,
                                                    static_cast<T*>(y), stats_out, stats_in, (int)full_dim);
  else
    polynorm_kernel<T, 16 / sizeof(T)><<<rows, threads, 0, st>>>(
        xp, up_p, in_stride, static_cast<const T*>(w), static_cast<const T*>(b), eps, (int)dim,
        static_cast<T*>(y), stats_out, stats_in, (int)full_dim);
  return check_launch("polynorm");
}

// ---------------------------------------------------------------------------
// RMSNorm with optional residual add and embedding gather.
//   mode 0: y = rms(x)·w
//   mode 1: h = T(h + delta); y = rms(h)·w      (h in/out)
//   mode 2: h = table[token]; y = rms(h)·w
// ---------------------------------------------------------------------------
template <typename T, int V>
__global__ void rms_norm_kernel(int mode, const T* __restrict__ x, T* h, const T* __restrict__ delta,
                                const int32_t* __restrict__ token, int64_t vocab,
                                const T* __restrict__ w, float eps, int dim, T* __restrict__ y) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const T* src;
  if (mode == 2) {
    int64_t t = token[row];
    if (t < 0 || t >= vocab) t = 0;  // out-of-range ids read row 0 (documented)
    src = x + t * (int64_t)dim;
  } else if (mode == 1) {
    src = h + row * (int64_t)dim;
  } else {
    src = x + row * (int64_t)dim;
  }
  float acc[1] = {0.f};
  for (int i = threadIdx.x * V; i < dim; i += blockDim.x * V) {
    float v[V];
    load_vec<T, V>(src + i, v);
    if (mode == 1) {
      float d[V];
      load_vec<T, V>(delta + row * (int64_t)dim + i, d);
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = round_through<T>(v[j] + d[j]);
    }
#pragma unroll
    for (int j = 0; j < V; ++j) acc[0] += v[j] * v[j];
  }
  block_sum<1>(acc, scratch);
  const float inv = rsqrtf(acc[0] / (float)dim + eps);
  for (int i = threadIdx.x * V; i < dim; i += blockDim.x * V) {
    float v[V], wv[V], o[V];
    load_vec<T, V>(src + i, v);
    if (mode == 1) {
      float d[V];
      load_vec<T, V>(delta + row * (int64_t)dim + i, d);
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = round_through<T>(v[j] + d[j]);
    }
    load_vec<T, V>(w + i, wv);
#pragma unroll
    for (int j = 0; j < V; ++j) o[j] = v[j] * inv * wv[j];
    store_vec<T, V>(y + row * (int64_t)dim + i, o);
    if (mode != 0) store_vec<T, V>(h + row * (int64_t)dim + i, v);
  }
}

template <typename T>
int launch_rms(int mode, const void* x, void* h, const void* delta, const int32_t* token,
               int64_t vocab, const void* w, float eps, int64_t rows, int64_t dim, void* y,
               cudaStream_t st) {
  const int V = vec_width<T>(dim, {x, h, delta, w, y}, {});
  const int threads = pick_threads(ceil_div(dim, V));
  if (V == 1)
    rms_norm_kernel<T, 1><<<rows, threads, 0, st>>>(
        mode, static_cast<const T*>(x), static_cast<T*>(h), static_cast<const T*>(delta), token,
        vocab, static_cast<const T*>(w), eps, (int)dim, static_cast<T*>(y));
  else
    rms_norm_kernel<T, 16 / sizeof(T)><<<rows, threads, 0, st>>>(
        mode, static_cast<const T*>(x), static_cast<T*>(h), static_cast<const T*>(delta), token,
        vocab, static_cast<const T*>(w), eps, (int)dim, static_cast<T*>(y));
  return check_launch("rms_norm");
}

// ---------------------------------------------------------------------------
// GDA post reduction (gda.py:131-192): one warp per (b, h_o, s) row of C
// channels. λ index: 0 (per-layer scalar), h_o/gr (per noise group) or h_o.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void gda_post_kernel(const T* __restrict__ o_base, int64_t o_bstride,
                                const T* __restrict__ n_base, int64_t n_bstride,
                                int64_t head_stride, const T* __restrict__ w,
                                const float* __restrict__ lam, int lam_mode, float out_scale,
                                float eps, int64_t rows, int q_origin, int gr, int S, int C,
                                T* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t per_b = (int64_t)q_origin * S;
  const int64_t b = row / per_b;
  const int64_t r = row - b * per_b;
  const int h_o = (int)(r / S);
  const int s = (int)(r - (int64_t)h_o * S);
  const T* op = o_base + b * o_bstride + h_o * head_stride + (int64_t)s * C;
  const T* np = n_base + b * n_bstride + (h_o / gr) * head_stride + (int64_t)s * C;
  T* yp = y + row * (int64_t)C;
  const float l = lam[lam_mode == 0 ? 0 : (lam_mode == 1 ? h_o / gr : h_o)];
  float ssq = 0.f;
  for (int c = lane; c < C; c += 32) {
    float d = to_f<T>(op[c]) - l * to_f<T>(np[c]);
    ssq += d * d;
  }
  ssq = warp_sum(ssq);
  const float inv = rsqrtf(ssq / (float)C + eps);
  for (int c = lane; c < C; c += 32) {
    float d = to_f<T>(op[c]) - l * to_f<T>(np[c]);
    yp[c] = from_f<T>(d * inv * to_f<T>(w[c]) * out_scale);
  }
}

// ---------------------------------------------------------------------------
// Greedy argmax: first index of the maximum (NaN ranks below everything).
// ---------------------------------------------------------------------------
struct Best {
  float v;
  int32_t i;
};

__device__ __forceinline__ Best better(Best a, Best b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ __forceinline__ Best warp_best(Best x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best y{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
    x = better(x, y);
  }
  return x;
}

template <typename T>
__global__ void argmax_partial_kernel(const T* __restrict__ x, int64_t n, Best* __restrict__ part) {
  __shared__ Best sm[32];
  pdl_trigger();
  Best best{-INFINITY, 0x7fffffff};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f<T>(x[i]);
    if (isnan(v)) v = -INFINITY;
    best = better(best, Best{v, (int32_t)i});
  }
  best = warp_best(best);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sm[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = lane < (int)(blockDim.x >> 5) ? sm[lane] : Best{-INFINITY, 0x7fffffff};
    best = warp_best(best);
    if (lane == 0) part[blockIdx.x] = best;
  }
}

__global__ void argmax_final_kernel(const Best* __restrict__ part, int nparts,
                                    int32_t* __restrict__ out) {
  Best best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < nparts; i += 32) best = better(best, part[i]);
  best = warp_best(best);
  if (threadIdx.x == 0) out[0] = best.i == 0x7fffffff ? 0 : best.i;
}

// Token from a combined argmax key (see argmax_key_out of motif_linear_fused).
__global__ void argmax_key_decode_kernel(const long long* __restrict__ key, int32_t* __restrict__ token,
                                         int32_t* __restrict__ pos_len) {
  const unsigned long long k = (unsigned long long)key[0] ^ 0x8000000000000000ull;
  token[0] = k == 0 ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
  if (pos_len) {
    pos_len[0] += 1;
    pos_len[1] += 1;
  }
}

// The tensor-parallel greedy/sampled token over peer memory. Each rank's key (value bits << 32 |
// (2^32 - 1 - row), as the lm_head epilogue or motif_sample_key writes it, sign-flipped) is
// re-packed with a step number in bits 24..31 of its low word — (value bits << 32) | number << 24 |
// (2^24 - 1 - row) — and stored, one 8-byte element, into slot [parity * world + rank] of every
// rank's key area. Keys of one step all carry the same number, so the largest packed key is still
// the largest value at its first row. Each rank then reads its own area until all `world` slots
// carry this step's number (bounded), and decodes the largest. number = pos % 255 + 1 is never 0
// (a zeroed area) and a slot is rewritten every second step, so a stale key never matches.
struct KeySlots {
  long long* p[8];
};
__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr unsigned long long kKeyWaitNs = 2000ull * 1000 * 1000;

__global__ void argmax_key_exchange_kernel(const long long* __restrict__ key, KeySlots slots, int world, int rank,
                                           const int32_t* __restrict__ pos_dev, int32_t* __restrict__ token,
                                           int32_t* __restrict__ pos_len, int32_t* __restrict__ err) {
  const int i = threadIdx.x;
  const int pos = pos_dev[0];
  const unsigned long long number = (unsigned long long)(((pos % 255) + 255) % 255 + 1);
  const int par = pos & 1;
  const unsigned long long k = (unsigned long long)key[0] ^ 0x8000000000000000ull;
  const uint32_t row = 0xFFFFFFFFu - (uint32_t)k;
  const unsigned long long packed =
      k == 0 ? (number << 24) : ((k & 0xFFFFFFFF00000000ull) | (number << 24) | (0xFFFFFFu - (row & 0xFFFFFFu)));
  if (i < world) {
    long long* dst = slots.p[i] + par * world + rank;
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(dst), "l"((long long)packed) : "memory");
  }
  unsigned long long v = 0;
  if (i < world) {
    const long long* src = slots.p[rank] + par * world + i;
    long long x;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(x) : "l"(src) : "memory");
    if ((((unsigned long long)x >> 24) & 0xFFu) != number) {
      const unsigned long long t0 = global_timer_ns();
      do {
        __nanosleep(64);
        asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(x) : "l"(src) : "memory");
        if (global_timer_ns() - t0 > kKeyWaitNs) {
          if (err) atomicExch(err, 2);
          break;
        }
      } while ((((unsigned long long)x >> 24) & 0xFFu) != number);
    }
    v = (unsigned long long)x;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  if (i == 0) {
    const uint32_t field = (uint32_t)(v & 0xFFFFFFu);
    token[0] = ((v >> 32) == 0 && field == 0) ? 0 : (int32_t)(0xFFFFFFu - field);
    if (pos_len) {
      pos_len[0] += 1;
      pos_len[1] += 1;
    }
  }
}

constexpr int kArgmaxThreads = 256;
int argmax_parts(int64_t n) {
  int64_t p = ceil_div(n, kArgmaxThreads * 8);
  if (p < 1) p = 1;
  if (p > 256) p = 256;
  return (int)p;
}

}  // namespace
}  // namespace motif

using namespace motif;

extern "C" {

int motif_polynorm(int dtype, const void* x, const void* weight, const void* bias, float eps,
                   int64_t rows, int64_t dim, void* y, void* stream) {
  MOTIF_REQUIRE(x && weight && bias && y, MOTIF_ERR_NULL, "polynorm: null pointer");
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim < (1ll << 31), MOTIF_ERR_BAD_SHAPE,
                "polynorm: rows=%lld dim=%lld", (long long)rows, (long long)dim);
  if (rows == 0) return MOTIF_OK;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_polynorm<T>(x, nullptr, dim, weight, bias, eps, rows, dim, y, as_stream(stream)));
  return MOTIF_OK;
}

int motif_polynorm_mul(int dtype, const void* gate, const void* up, int64_t in_stride,
                       const void* weight, const void* bias, float eps, int64_t rows, int64_t dim,
                       void* y, void* stream) {
  MOTIF_REQUIRE(gate && up && weight && bias && y, MOTIF_ERR_NULL, "polynorm_mul: null pointer");
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim < (1ll << 31) && in_stride >= dim, MOTIF_ERR_BAD_SHAPE,
                "polynorm_mul: rows=%lld dim=%lld stride=%lld", (long long)rows, (long long)dim,
                (long long)in_stride);
  if (rows == 0) return MOTIF_OK;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_polynorm<T>(gate, up, in_stride, weight, bias, eps, rows, dim, y, as_stream(stream)));
  return MOTIF_OK;
}

int motif_polynorm_row_stats(int dtype, const void* x, int64_t in_stride, int64_t rows, int64_t dim, float* stats,
                             void* stream) {
  MOTIF_REQUIRE(x && stats, MOTIF_ERR_NULL, "polynorm_row_stats: null pointer");
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim < (1ll << 31) && in_stride >= dim, MOTIF_ERR_BAD_SHAPE,
                "polynorm_row_stats: rows=%lld dim=%lld stride=%lld", (long long)rows, (long long)dim,
                (long long)in_stride);
  if (rows == 0) return MOTIF_OK;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_polynorm<T>(x, nullptr, in_stride, nullptr, nullptr, 0.f, rows, dim,
                                                           nullptr, as_stream(stream), stats));
  return MOTIF_OK;
}

int motif_polynorm_mul_stats(int dtype, const void* gate, const void* up, int64_t in_stride, const void* weight,
                             const void* bias, float eps, int64_t rows, int64_t dim, const float* stats,
                             int64_t full_dim, void* y, void* stream) {
  MOTIF_REQUIRE(gate && up && weight && bias && stats && y, MOTIF_ERR_NULL, "polynorm_mul_stats: null pointer");
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim < (1ll << 31) && in_stride >= dim && full_dim >= dim &&
                    full_dim < (1ll << 31),
                MOTIF_ERR_BAD_SHAPE, "polynorm_mul_stats: rows=%lld dim=%lld stride=%lld full_dim=%lld",
                (long long)rows, (long long)dim, (long long)in_stride, (long long)full_dim);
  if (rows == 0) return MOTIF_OK;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_polynorm<T>(gate, up, in_stride, weight, bias, eps, rows, dim, y,
                                                           as_stream(stream), nullptr, stats, full_dim));
  return MOTIF_OK;
}

int motif_rms_norm(int dtype, const void* x, const void* w, float eps, int64_t rows, int64_t dim,
                   void* y, void* stream) {
  MOTIF_REQUIRE(x && w && y, MOTIF_ERR_NULL, "rms_norm: null pointer");
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "rms_norm: bad shape");
  if (rows == 0) return MOTIF_OK;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_rms<T>(0, x, nullptr, nullptr, nullptr, 0, w, eps, rows, dim, y, as_stream(stream)));
  return MOTIF_OK;
}

int motif_add_rms_norm(int dtype, void* h, const void* delta, const void* w, float eps,
                       int64_t rows, int64_t dim, void* y, void* stream) {
  MOTIF_REQUIRE(h && delta && w && y, MOTIF_ERR_NULL, "add_rms_norm: null pointer");
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "add_rms_norm: bad shape");
  if (rows == 0) return MOTIF_OK;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_rms<T>(1, nullptr, h, delta, nullptr, 0, w, eps, rows, dim, y, as_stream(stream)));
  return MOTIF_OK;
}

int motif_embed_rms_norm(int dtype, const int32_t* token_dev, const void* table, int64_t vocab,
                         int64_t dim, const void* w, float eps, void* h, void* y, void* stream) {
  MOTIF_REQUIRE(token_dev && table && w && h && y, MOTIF_ERR_NULL, "embed_rms_norm: null pointer");
  MOTIF_REQUIRE(vocab > 0 && dim > 0 && dim < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "embed_rms_norm: bad shape");
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_rms<T>(2, table, h, nullptr, token_dev, vocab, w, eps, 1, dim, y, as_stream(stream)));
  return MOTIF_OK;
}

int motif_embed_rms_norm_rows(int dtype, const int32_t* tokens_dev, int64_t rows, const void* table, int64_t vocab,
                              int64_t dim, const void* w, float eps, void* h, void* y, void* stream) {
  MOTIF_REQUIRE(tokens_dev && table && w && h && y, MOTIF_ERR_NULL, "embed_rms_norm_rows: null pointer");
  MOTIF_REQUIRE(rows >= 0 && rows < (1ll << 31) && vocab > 0 && dim > 0 && dim < (1ll << 31), MOTIF_ERR_BAD_SHAPE,
                "embed_rms_norm_rows: bad shape");
  if (rows == 0) return MOTIF_OK;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_rms<T>(2, table, h, nullptr, tokens_dev, vocab, w, eps, rows, dim, y, as_stream(stream)));
  return MOTIF_OK;
}

static int gda_common(int dtype, const void* o_base, int64_t o_bstride, const void* n_base,
                      int64_t n_bstride, const void* subln_w, const float* lam, int64_t lam_len,
                      float lambda_init, int64_t B, int64_t q_groups, int64_t gr, int64_t S,
                      int64_t C, float eps, void* y, void* stream) {
  const int64_t q_origin = q_groups * gr;
  int lam_mode;
  if (lam_len == 1) lam_mode = 0;
  else if (lam_len == q_groups) lam_mode = 1;
  else if (lam_len == q_origin) lam_mode = 2;
  else return fail(MOTIF_ERR_BAD_SHAPE, "gda_post: lambda_full has %lld values; expected 1, %lld or %lld",
                   (long long)lam_len, (long long)q_groups, (long long)q_origin);
  const int64_t rows = B * q_origin * S;
  if (rows == 0) return MOTIF_OK;
  const int warps = 8;
  const int64_t blocks = ceil_div(rows, warps);
  const float out_scale = 1.0f - lambda_init;
  cudaStream_t st = as_stream(stream);
  MOTIF_DISPATCH_FLOAT(dtype, T, {
    gda_post_kernel<T><<<blocks, warps * 32, 0, st>>>(
        static_cast<const T*>(o_base), o_bstride, static_cast<const T*>(n_base), n_bstride, S * C,
        static_cast<const T*>(subln_w), lam, lam_mode, out_scale, eps, rows, (int)q_origin, (int)gr,
        (int)S, (int)C, static_cast<T*>(y));
  });
  return check_launch("gda_post");
}

int motif_gda_post_split(int dtype, const void* attn_o, const void* attn_n, const void* subln_w,
                         const float* lambda_full, int64_t lambda_len, float lambda_init,
                         int64_t batch, int64_t q_groups, int64_t gr, int64_t seq, int64_t channels,
                         float eps, void* y, void* stream) {
  MOTIF_REQUIRE(attn_o && attn_n && subln_w && lambda_full && y, MOTIF_ERR_NULL, "gda_post_split: null pointer");
  MOTIF_REQUIRE(batch >= 0 && q_groups > 0 && gr > 0 && seq >= 0 && channels > 0 && channels < (1 << 30),
                MOTIF_ERR_BAD_SHAPE, "gda_post_split: bad shape");
  const int64_t q_origin = q_groups * gr;
  return gda_common(dtype, attn_o, q_origin * seq * channels, attn_n, q_groups * seq * channels,
                    subln_w, lambda_full, lambda_len, lambda_init, batch, q_groups, gr, seq,
                    channels, eps, y, stream);
}

int motif_gda_post(int dtype, const void* merged, const void* subln_w, const float* lambda_full,
                   int64_t lambda_len, float lambda_init, int64_t batch, int64_t q_groups,
                   int64_t gr, int64_t seq, int64_t channels, float eps, void* y, void* stream) {
  MOTIF_REQUIRE(merged && subln_w && lambda_full && y, MOTIF_ERR_NULL, "gda_post: null pointer");
  MOTIF_REQUIRE(batch >= 0 && q_groups > 0 && gr > 0 && seq >= 0 && channels > 0 && channels < (1 << 30),
                MOTIF_ERR_BAD_SHAPE, "gda_post: bad shape");
  const int64_t q_origin = q_groups * gr;
  const int64_t bstride = (q_origin + q_groups) * seq * channels;
  size_t esz = dtype == MOTIF_F32 ? 4 : 2;
  const void* n_base = static_cast<const char*>(merged) + q_origin * seq * channels * esz;
  return gda_common(dtype, merged, bstride, n_base, bstride, subln_w, lambda_full, lambda_len,
                    lambda_init, batch, q_groups, gr, seq, channels, eps, y, stream);
}

size_t motif_argmax_workspace_bytes(int64_t n) { return sizeof(Best) * (size_t)argmax_parts(n); }

int motif_argmax_key_decode(const int64_t* key, int32_t* token, int32_t* pos_len_inc, void* stream) {
  MOTIF_REQUIRE(key && token, MOTIF_ERR_NULL, "argmax_key_decode: null pointer");
  argmax_key_decode_kernel<<<1, 1, 0, as_stream(stream)>>>(reinterpret_cast<const long long*>(key), token, pos_len_inc);
  return check_launch("argmax_key_decode");
}

int motif_argmax_key_exchange(const int64_t* key, int64_t* const* slots, int world, int rank, const int32_t* pos_dev,
                              int32_t* token, int32_t* pos_len_inc, int32_t* err, void* stream) {
  MOTIF_REQUIRE(key && slots && pos_dev && token, MOTIF_ERR_NULL, "argmax_key_exchange: null pointer");
  MOTIF_REQUIRE(world >= 1 && world <= 8 && rank >= 0 && rank < world, MOTIF_ERR_BAD_CONTRACT,
                "argmax_key_exchange: rank %d of world %d (1..8)", rank, world);
  KeySlots ks{};
  for (int r = 0; r < world; ++r) {
    MOTIF_REQUIRE(slots[r] && reinterpret_cast<uintptr_t>(slots[r]) % 8 == 0, MOTIF_ERR_NULL,
                  "argmax_key_exchange: key area of rank %d", r);
    ks.p[r] = reinterpret_cast<long long*>(slots[r]);
  }
  argmax_key_exchange_kernel<<<1, 32, 0, as_stream(stream)>>>(reinterpret_cast<const long long*>(key), ks, world,
                                                               rank, pos_dev, token, pos_len_inc, err);
  return check_launch("argmax_key_exchange");
}

int motif_argmax(int dtype, const void* logits, int64_t n, int32_t* out_index, void* workspace,
                 size_t workspace_bytes, void* stream) {
  MOTIF_REQUIRE(logits && out_index && workspace, MOTIF_ERR_NULL, "argmax: null pointer");
  MOTIF_REQUIRE(n > 0 && n < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "argmax: n=%lld", (long long)n);
  const int parts = argmax_parts(n);
  MOTIF_REQUIRE(workspace_bytes >= sizeof(Best) * (size_t)parts, MOTIF_ERR_WORKSPACE,
                "argmax: workspace %zu < %zu", workspace_bytes, sizeof(Best) * (size_t)parts);
  cudaStream_t st = as_stream(stream);
  Best* part = static_cast<Best*>(workspace);
  MOTIF_DISPATCH_FLOAT(dtype, T, {
    argmax_partial_kernel<T><<<parts, kArgmaxThreads, 0, st>>>(static_cast<const T*>(logits), n, part);
  });
  argmax_final_kernel<<<1, 32, 0, st>>>(part, parts, out_index);
  return check_launch("argmax");
}

}  // extern "C"
