// Sampling for the decode and speculative paths.
//
// Temperature sampling is Gumbel-max: token = argmax_i (l_i / T + g_i) with g_i = −log(−log u_i)
// and u_i uniform, which draws exactly from softmax(l / T) (top-p 1.0, the reference's
// speculative configuration). T = 0 is the greedy argmax (first index of the maximum). The
// uniforms come from Philox-4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011), keyed by a 64-bit seed and counted by (element, position, row,
// stream), so a replayed CUDA graph draws fresh numbers at every position.
//
// The speculative acceptance follows the rejection rule of speculative sampling (the reference's
// MotifSpeculativeDecoding: accept draft token x_i with probability min(1, p_i(x_i) / q_i(x_i)),
// on the first rejection draw from the residual max(0, p_i − q_i) renormalised, and after K
// acceptances draw the bonus token from p_K). At T = 0 it reduces to "accept while the draft
// equals the target's argmax".
#include <cmath>

#include "common.cuh"

namespace motif {
namespace {

__device__ __forceinline__ uint4 philox4x32(uint4 c, uint2 k) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u, kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k.x += kW0;
      k.y += kW1;
    }
    const uint32_t hi0 = __umulhi(kM0, c.x), lo0 = kM0 * c.x;
    const uint32_t hi1 = __umulhi(kM1, c.z), lo1 = kM1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  return c;
}

// Uniform in (0, 1) from 24 random bits (never 0 or 1, so both logs are finite).
__device__ __forceinline__ float uniform01(uint32_t bits) { return ((bits >> 8) + 0.5f) * (1.0f / 16777216.0f); }

__device__ __forceinline__ float gumbel(uint64_t seed, uint32_t i, uint32_t pos, uint32_t row, uint32_t stream) {
  const uint4 r = philox4x32(make_uint4(i, pos, row, stream), make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
  return -__logf(-__logf(uniform01(r.x)));
}

// Order-preserving 64-bit key: larger value wins, then the smaller index.
__device__ __forceinline__ unsigned long long sample_key(float v, uint32_t i) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (0xFFFFFFFFu - i);
}
__device__ __forceinline__ uint32_t key_index(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull); }

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  v = lane < nw ? sm[lane] : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

__device__ __forceinline__ float block_reduce(float v, float* sm, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = is_max ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  v = lane < nw ? sm[lane] : (is_max ? -INFINITY : 0.f);
  return is_max ? warp_max(v) : warp_sum(v);
}

constexpr int kSampleThreads = 1024;

// One CTA per row: token = argmax(l / T + g) (T > 0) or argmax(l).
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const __half* __restrict__ logits, int64_t stride,
                                                                int n, float inv_t, uint64_t seed,
                                                                const int32_t* __restrict__ pos_dev, int pos_host,
                                                                uint32_t stream_id, int32_t* __restrict__ tokens,
                                                                int32_t* __restrict__ pos_len_inc) {
  __shared__ unsigned long long sm[32];
  const int row = blockIdx.x;
  const __half* l = logits + row * stride;
  const uint32_t pos = (uint32_t)(pos_dev ? *pos_dev : pos_host);
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = __half2float(l[i]);
    if (isnan(v)) v = -INFINITY;
    if (inv_t > 0.f) v = v * inv_t + gumbel(seed, (uint32_t)i, pos, (uint32_t)row, stream_id);
    const unsigned long long k = sample_key(v, (uint32_t)i);
    best = k > best ? k : best;
  }
  best = block_max_u64(best, sm);
  if (threadIdx.x == 0) {
    tokens[row] = best ? (int32_t)key_index(best) : 0;
    if (pos_len_inc && row == 0) {
      pos_len_inc[0] += 1;
      pos_len_inc[1] += 1;
    }
  }
}

// One shard of a vocabulary split over tensor-parallel ranks: the largest key of (l / T + g) over
// this shard's n logits, the noise drawn for the GLOBAL index row_offset + i (the same numbers
// one GPU draws for the whole row), written as a signed int64 so an int64 MAX all-reduce over
// the ranks yields the key of the whole row.
__global__ void __launch_bounds__(kSampleThreads) sample_key_kernel(const __half* __restrict__ logits, int n,
                                                                    float inv_t, uint64_t seed,
                                                                    const int32_t* __restrict__ pos_dev, int pos_host,
                                                                    uint32_t stream_id, uint32_t row_offset,
                                                                    long long* __restrict__ key_out) {
  __shared__ unsigned long long sm[32];
  const uint32_t pos = (uint32_t)(pos_dev ? *pos_dev : pos_host);
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = __half2float(logits[i]);
    if (isnan(v)) v = -INFINITY;
    const uint32_t gi = row_offset + (uint32_t)i;
    if (inv_t > 0.f) v = v * inv_t + gumbel(seed, gi, pos, 0u, stream_id);
    const unsigned long long k = sample_key(v, gi);
    best = k > best ? k : best;
  }
  best = block_max_u64(best, sm);
  if (threadIdx.x == 0) *key_out = (long long)(best ^ 0x8000000000000000ull);
}

// Speculative acceptance over K draft tokens: p rows 0..K (target), q rows 0..K-1 (draft).
// out[0] = accepted count n, out[1] = the token that follows them.
constexpr int kMaxDraft = 16;
__global__ void __launch_bounds__(kSampleThreads) spec_accept_kernel(const __half* __restrict__ p, const __half* __restrict__ q,
                                                                     int64_t stride, const int32_t* __restrict__ draft,
                                                                     int K, int n, float inv_t, uint64_t seed,
                                                                     const int32_t* __restrict__ pos_dev, int pos_host,
                                                                     int32_t* __restrict__ out) {
  __shared__ float smf[32];
  __shared__ unsigned long long smk[32];
  __shared__ float s_m[2 * kMaxDraft + 1], s_z[2 * kMaxDraft + 1];
  __shared__ int s_arg[kMaxDraft + 1];
  __shared__ int s_n;
  const uint32_t pos = (uint32_t)(pos_dev ? *pos_dev : pos_host);
  const bool greedy = !(inv_t > 0.f);
  // row statistics: max and Σ exp(l/T − max) of every p and q row (argmax of the p rows)
  const int nrows = greedy ? K + 1 : 2 * K + 1;  // the greedy rule needs only the target's argmaxes
  for (int r = 0; r < nrows; ++r) {
    const __half* l = r <= K ? p + r * stride : q + (r - K - 1) * stride;
    float m = -INFINITY;
    unsigned long long best = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float v = __half2float(l[i]);
      if (isnan(v)) v = -INFINITY;
      if (r <= K && greedy) {
        const unsigned long long k = sample_key(v, (uint32_t)i);
        best = k > best ? k : best;
      }
      m = fmaxf(m, v * (greedy ? 1.f : inv_t));
    }
    m = block_reduce(m, smf, true);
    if (r <= K && greedy) best = block_max_u64(best, smk);
    float z = 0.f;
    if (!greedy)
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = __half2float(l[i]) * inv_t;
        z += (v == -INFINITY || isnan(v)) ? 0.f : __expf(v - m);
      }
    z = block_reduce(z, smf, false);
    if (threadIdx.x == 0) {
      s_m[r] = m;
      s_z[r] = z;
      if (r <= K) s_arg[r] = greedy ? (best ? (int)key_index(best) : 0) : 0;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = K;
    for (int i = 0; i < K; ++i) {
      const int x = min(max(draft[i], 0), n - 1);
      bool ok;
      if (greedy) {
        ok = x == s_arg[i];
      } else {
        const float lp = __half2float(p[i * stride + x]) * inv_t, lq = __half2float(q[i * stride + x]) * inv_t;
        const float pp = __expf(lp - s_m[i]) / s_z[i], qq = __expf(lq - s_m[K + 1 + i]) / s_z[K + 1 + i];
        const uint4 rr = philox4x32(make_uint4((uint32_t)i, pos, 0xACCE97u, 1u),
                                    make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
        ok = uniform01(rr.x) * qq < pp;
      }
      if (!ok) {
        acc = i;
        break;
      }
    }
    s_n = acc;
  }
  __syncthreads();
  const int a = s_n;
  if (greedy) {
    if (threadIdx.x == 0) {
      out[0] = a;
      out[1] = s_arg[a];
    }
    return;
  }
  // the next token: from p_K after K acceptances, else from max(0, p_a − q_a) (p_a if that is empty)
  const __half* lp = p + a * stride;
  const __half* lq = a < K ? q + a * stride : nullptr;
  unsigned long long best = 0, best_p = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float g = gumbel(seed, (uint32_t)i, pos, 0x5E5Du + (uint32_t)a, 2u);
    const float vp = __half2float(lp[i]) * inv_t;
    const float pp = isnan(vp) ? 0.f : __expf(vp - s_m[a]) / s_z[a];
    if (pp > 0.f) {
      const unsigned long long kp = sample_key(__logf(pp) + g, (uint32_t)i);
      best_p = kp > best_p ? kp : best_p;
    }
    float w = pp;
    if (lq) {
      const float vq = __half2float(lq[i]) * inv_t;
      w = pp - (isnan(vq) ? 0.f : __expf(vq - s_m[K + 1 + a]) / s_z[K + 1 + a]);
    }
    if (w > 0.f) {
      const unsigned long long k = sample_key(__logf(w) + g, (uint32_t)i);
      best = k > best ? k : best;
    }
  }
  best = block_max_u64(best, smk);
  best_p = block_max_u64(best_p, smk);
  if (threadIdx.x == 0) {
    out[0] = a;
    out[1] = (int32_t)key_index(best ? best : best_p);
  }
}

}  // namespace
}  // namespace motif

using namespace motif;

extern "C" {

int motif_sample(const void* logits, int64_t rows, int64_t n, int64_t row_stride, float temperature, uint64_t seed,
                 const int32_t* pos_dev, int64_t pos_host, uint32_t stream_id, int32_t* tokens,
                 void* pos_len_inc, void* stream) {
  MOTIF_REQUIRE(logits && tokens, MOTIF_ERR_NULL, "sample: null pointer");
  MOTIF_REQUIRE(rows >= 1 && rows < 65536 && n > 0 && n < (1ll << 31) && row_stride >= n, MOTIF_ERR_BAD_SHAPE,
                "sample: rows=%lld n=%lld stride=%lld", (long long)rows, (long long)n, (long long)row_stride);
  MOTIF_REQUIRE(temperature >= 0.f, MOTIF_ERR_BAD_CONTRACT, "sample: temperature %f", temperature);
  sample_kernel<<<(unsigned)rows, kSampleThreads, 0, as_stream(stream)>>>(
      static_cast<const __half*>(logits), row_stride, (int)n, temperature > 0.f ? 1.f / temperature : 0.f, seed,
      pos_dev, (int)pos_host, stream_id, tokens, static_cast<int32_t*>(pos_len_inc));
  return check_launch("sample");
}

int motif_sample_key(const void* logits, int64_t n, float temperature, uint64_t seed, const int32_t* pos_dev,
                     int64_t pos_host, uint32_t stream_id, int64_t row_offset, int64_t* key_out, void* stream) {
  MOTIF_REQUIRE(logits && key_out, MOTIF_ERR_NULL, "sample_key: null pointer");
  MOTIF_REQUIRE(n > 0 && row_offset >= 0 && row_offset + n <= 0xFFFFFFFFll, MOTIF_ERR_BAD_SHAPE,
                "sample_key: n=%lld row_offset=%lld", (long long)n, (long long)row_offset);
  MOTIF_REQUIRE(temperature >= 0.f, MOTIF_ERR_BAD_CONTRACT, "sample_key: temperature %f", temperature);
  sample_key_kernel<<<1, kSampleThreads, 0, as_stream(stream)>>>(
      static_cast<const __half*>(logits), (int)n, temperature > 0.f ? 1.f / temperature : 0.f, seed, pos_dev,
      (int)pos_host, stream_id, (uint32_t)row_offset, reinterpret_cast<long long*>(key_out));
  return check_launch("sample_key");
}

int motif_speculative_accept(const void* p_logits, const void* q_logits, int64_t row_stride,
                             const int32_t* draft_tokens, int64_t k, int64_t n, float temperature, uint64_t seed,
                             const int32_t* pos_dev, int64_t pos_host, int32_t* out, void* stream) {
  MOTIF_REQUIRE(p_logits && draft_tokens && out && (q_logits || temperature == 0.f), MOTIF_ERR_NULL,
                "speculative_accept: null pointer");
  MOTIF_REQUIRE(k >= 1 && k <= kMaxDraft && n > 0 && n < (1ll << 31) && row_stride >= n, MOTIF_ERR_BAD_SHAPE,
                "speculative_accept: k=%lld (1..%d) n=%lld", (long long)k, kMaxDraft, (long long)n);
  MOTIF_REQUIRE(temperature >= 0.f, MOTIF_ERR_BAD_CONTRACT, "speculative_accept: temperature %f", temperature);
  spec_accept_kernel<<<1, kSampleThreads, 0, as_stream(stream)>>>(
      static_cast<const __half*>(p_logits), static_cast<const __half*>(q_logits), row_stride, draft_tokens, (int)k,
      (int)n, temperature > 0.f ? 1.f / temperature : 0.f, seed, pos_dev, (int)pos_host, out);
  return check_launch("speculative_accept");
}

}  // extern "C"
