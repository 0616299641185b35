// Shared-QK dual-V decode attention, split-KV ("flash-decode") on B200.
//
// One CTA owns one (batch, kv head) and one contiguous chunk of KV positions,
// and serves every query head that reads that kv head: the GQA heads of the
// generic op, or — in the fused GDA layer path — the gr origin heads (slot
// k1) plus the noise head (slot k2) of one group. Each cache row (k1, k2, v1,
// v2) is therefore read from HBM exactly once per layer.
//
// Inside a CTA, 8 warps each take 4 consecutive positions per round (16
// independent loads per lane in flight), a lane owns D/32 channels, scores
// are warp all-reduced, and the online softmax (base-2, scale·log2e folded
// into q) updates two V accumulators with one weight. Warps merge through
// shared memory; splits merge in a second kernel (plain, or fused with the
// GDA post reduction).
//
// Packed caches (bits 4/8, MLX affine triples) are dequantized in registers:
// a lane's D/32 channels sit in one uint32 and one scale/bias group, the same
// lane→word contract the reference enforces (attention.py:565-608).
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "kvquant.cuh"
#include "tma.cuh"

namespace motif {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kPosPerWarp = 4;
constexpr int kRoundPositions = kAttnWarps * kPosPerWarp;  // 32
constexpr int kMinChunk = 32;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  const void* q;
  int64_t q_bstride;  // elements between batches of q
  int na;             // A heads per kv head (runtime, <= MAXA)
  int nb_base;        // head index of the B head of kv head 0
  int h_out;          // heads per batch in y / workspace indexing
  const void* kA;
  const void* kB;
  const void* v1;
  const void* v2;
  const void* kA_s;
  const void* kA_b;
  const void* kB_s;
  const void* kB_b;
  const void* v1_s;
  const void* v1_b;
  const void* v2_s;
  const void* v2_b;
  int h_kv;
  int64_t cap;
  int gs;
  int kv_len;
  const int32_t* kv_len_dev;
  float scale_log2;
  int force_partials;
  void* y;
  float* ws;
};

__device__ __forceinline__ void split_range(int kv_len, int nsplit, int split, int& p0, int& p1,
                                            int& n_active) {
  int chunk = (kv_len + nsplit - 1) / nsplit;
  if (chunk < kMinChunk) chunk = kMinChunk;
  n_active = (kv_len + chunk - 1) / chunk;
  p0 = split * chunk;
  p1 = min(kv_len, p0 + chunk);
}

template <typename T, int D, int BITS>
__device__ __forceinline__ void load_kv(const void* data, const void* sc, const void* bi, int64_t row,
                                        int lane, int gs, float (&out)[D / 32]) {
  constexpr int CPL = D / 32;
  if constexpr (BITS == 16) {
    load_vec<T, CPL>(static_cast<const T*>(data) + row * D + lane * CPL, out);
  } else {
    constexpr int EL = 32 / BITS;
    constexpr int WPR = D / EL;
    constexpr uint32_t MASK = (1u << BITS) - 1u;
    const int ch0 = lane * CPL;
    const uint32_t w = __ldg(static_cast<const uint32_t*>(data) + row * WPR + ch0 / EL);
    const int shift = (ch0 % EL) * BITS;
    const int64_t g = row * (D / gs) + ch0 / gs;
    const float s = to_f<T>(static_cast<const T*>(sc)[g]);
    const float b = to_f<T>(static_cast<const T*>(bi)[g]);
#pragma unroll
    for (int j = 0; j < CPL; ++j) out[j] = s * (float)((w >> (shift + j * BITS)) & MASK) + b;
  }
}

template <typename T, int D, int BITS, int MAXA, int NB>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(AttnArgs a) {
  constexpr int CPL = D / 32;
  constexpr int NH = MAXA + NB;
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int split = blockIdx.x, nsplit = gridDim.x;
  const int b = blockIdx.y / a.h_kv, hk = blockIdx.y % a.h_kv;
  const int kv_len = a.kv_len_dev ? *a.kv_len_dev : a.kv_len;
  int p0, p1, n_active;
  split_range(kv_len, nsplit, split, p0, p1, n_active);
  if (nsplit > 1 && split >= n_active) return;

  int head[NH];
  bool valid[NH];
#pragma unroll
  for (int h = 0; h < MAXA; ++h) {
    head[h] = hk * a.na + h;
    valid[h] = h < a.na;
  }
  if constexpr (NB > 0) {
    head[MAXA] = a.nb_base + hk;
    valid[MAXA] = true;
  }

  float q[NH][CPL];
  const T* qb = static_cast<const T*>(a.q) + (int64_t)b * a.q_bstride;
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    if (valid[h]) {
      load_vec<T, CPL>(qb + (int64_t)head[h] * D + lane * CPL, q[h]);
#pragma unroll
      for (int c = 0; c < CPL; ++c) q[h][c] *= a.scale_log2;
    } else {
#pragma unroll
      for (int c = 0; c < CPL; ++c) q[h][c] = 0.f;
    }
  }

  float m[NH], l[NH], o1[NH][CPL], o2[NH][CPL];
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) o1[h][c] = o2[h][c] = 0.f;
  }

  const int64_t row0 = ((int64_t)b * a.h_kv + hk) * a.cap;
  for (int base = p0 + warp * kPosPerWarp; base < p1; base += kRoundPositions) {
    float ka[kPosPerWarp][CPL], kb[kPosPerWarp][CPL], x1[kPosPerWarp][CPL], x2[kPosPerWarp][CPL];
#pragma unroll
    for (int u = 0; u < kPosPerWarp; ++u) {
      if (base + u < p1) {
        const int64_t r = row0 + base + u;
        load_kv<T, D, BITS>(a.kA, a.kA_s, a.kA_b, r, lane, a.gs, ka[u]);
        if constexpr (NB > 0) load_kv<T, D, BITS>(a.kB, a.kB_s, a.kB_b, r, lane, a.gs, kb[u]);
        load_kv<T, D, BITS>(a.v1, a.v1_s, a.v1_b, r, lane, a.gs, x1[u]);
        load_kv<T, D, BITS>(a.v2, a.v2_s, a.v2_b, r, lane, a.gs, x2[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kPosPerWarp; ++u) {
      if (base + u >= p1) break;
      float s[NH];
#pragma unroll
      for (int h = 0; h < MAXA; ++h) {
        float t = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) t += q[h][c] * ka[u][c];
        s[h] = t;
      }
      if constexpr (NB > 0) {
        float t = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) t += q[MAXA][c] * kb[u][c];
        s[MAXA] = t;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int h = 0; h < NH; ++h) s[h] += __shfl_xor_sync(0xffffffffu, s[h], o);
      }
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const float mn = fmaxf(m[h], s[h]);
        const float fac = exp2f(m[h] - mn);
        const float e = exp2f(s[h] - mn);
        m[h] = mn;
        l[h] = l[h] * fac + e;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          o1[h][c] = o1[h][c] * fac + e * x1[u][c];
          o2[h][c] = o2[h][c] * fac + e * x2[u][c];
        }
      }
    }
  }

  // ---- merge the warps' partial softmax states through shared memory ----
  extern __shared__ float smem[];
  float* sm_ml = smem;                          // [warp][h][2]
  float* sm_o = smem + kAttnWarps * NH * 2;     // [warp][h][2D]
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    if (lane == 0) {
      sm_ml[(warp * NH + h) * 2 + 0] = m[h];
      sm_ml[(warp * NH + h) * 2 + 1] = l[h];
    }
    float* dst = sm_o + (int64_t)(warp * NH + h) * 2 * D + lane * CPL;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      dst[c] = o1[h][c];
      dst[D + c] = o2[h][c];
    }
  }
  __syncthreads();
  const bool partial = nsplit > 1 || a.force_partials;
  for (int it = threadIdx.x; it < NH * 2 * D; it += kAttnThreads) {
    const int h = it / (2 * D);
    const int ch = it - h * 2 * D;
    if (h < MAXA && h >= a.na) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_ml[(w * NH + h) * 2]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float mw = sm_ml[(w * NH + h) * 2];
        if (mw == -INFINITY) continue;
        const float f = exp2f(mw - M);
        L += sm_ml[(w * NH + h) * 2 + 1] * f;
        O += sm_o[(int64_t)(w * NH + h) * 2 * D + ch] * f;
      }
    }
    int hh;
    if constexpr (NB > 0) hh = (h == MAXA) ? a.nb_base + hk : hk * a.na + h;
    else hh = hk * a.na + h;
    const int64_t bh = (int64_t)b * a.h_out + hh;
    if (partial) {
      float* p = a.ws + (bh * nsplit + split) * (2 * D + 2);
      p[2 + ch] = O;
      if (ch == 0) {
        p[0] = M;
        p[1] = L;
      }
    } else {
      static_cast<T*>(a.y)[bh * 2 * D + ch] = from_f<T>(L > 0.f ? O / L : 0.f);
    }
  }
}

constexpr int kMaxSplits = 64;

// Split weights of one head: f[s] = 2^(m_s − M), M = max_s m_s, and L = Σ l_s f[s],
// computed by one warp (two splits per lane) into shared memory.
__device__ __forceinline__ void split_weights(const float* __restrict__ base, int n_active, int stride,
                                              float* f_out, float* L_out, int lane) {
  // L2 loads: the partials may have been written by other CTAs of the same launch.
  const float m0 = lane < n_active ? __ldcg(base + lane * stride) : -INFINITY;
  const float m1 = lane + 32 < n_active ? __ldcg(base + (lane + 32) * stride) : -INFINITY;
  const float l0 = lane < n_active ? __ldcg(base + lane * stride + 1) : 0.f;
  const float l1 = lane + 32 < n_active ? __ldcg(base + (lane + 32) * stride + 1) : 0.f;
  const float M = warp_max(fmaxf(m0, m1));
  const float f0 = (M != -INFINITY && m0 != -INFINITY) ? exp2f(m0 - M) : 0.f;
  const float f1 = (M != -INFINITY && m1 != -INFINITY) ? exp2f(m1 - M) : 0.f;
  const float L = warp_sum(l0 * f0 + l1 * f1);
  f_out[lane] = f0;
  f_out[lane + 32] = f1;
  if (lane == 0) *L_out = L;
}

// Σ_s f[s] · o_s[ch] with independent loads (4 splits in flight per step).
__device__ __forceinline__ float merge_channel(const float* __restrict__ base, const float* f, int n_active,
                                              int stride, int ch) {
  float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
  int s = 0;
  for (; s + 4 <= n_active; s += 4) {
    o0 += f[s] * __ldcg(base + s * stride + 2 + ch);
    o1 += f[s + 1] * __ldcg(base + (s + 1) * stride + 2 + ch);
    o2 += f[s + 2] * __ldcg(base + (s + 2) * stride + 2 + ch);
    o3 += f[s + 3] * __ldcg(base + (s + 3) * stride + 2 + ch);
  }
  for (; s < n_active; ++s) o0 += f[s] * __ldcg(base + s * stride + 2 + ch);
  return (o0 + o1) + (o2 + o3);
}

// Merge split partials into the final (B, h_out, 2D) output; one CTA of 2D threads per row.
template <typename T, int D>
__global__ void attn_combine_kernel(const float* __restrict__ ws, int nsplit, int kv_len_host,
                                    const int32_t* __restrict__ kv_len_dev, T* __restrict__ y) {
  __shared__ float f_s[kMaxSplits];
  __shared__ float L_s;
  pdl_trigger();
  const int64_t bh = blockIdx.x;
  const int ch = threadIdx.x;
  const int kv_len = kv_len_dev ? *kv_len_dev : kv_len_host;
  int p0, p1, n_active;
  split_range(kv_len, nsplit, 0, p0, p1, n_active);
  constexpr int stride = 2 * D + 2;
  const float* base = ws + bh * nsplit * stride;
  if (threadIdx.x < 32) split_weights(base, n_active, stride, f_s, &L_s, threadIdx.x);
  __syncthreads();
  const float O = merge_channel(base, f_s, n_active, stride, ch);
  y[bh * 2 * D + ch] = from_f<T>(L_s > 0.f ? O / L_s : 0.f);
}

// Merge split partials of one GDA group and apply gda_post_split:
// out[h_o] = (o − λ·n) · rsqrt(mean d² + eps) · w · (1 − λ_init), with the
// attention outputs rounded through fp16 first (the reference materialises
// them as fp16 arrays between the two kernels). Run by a CTA of 2D threads.
template <int D, int GR>
__device__ __forceinline__ void gda_merge_group(const float* __restrict__ ws, int nsplit, int n_active, int g,
                                                int q_origin, const __half* __restrict__ subln_w,
                                                const float* __restrict__ lam, int lam_mode, float out_scale,
                                                float eps, __half* __restrict__ out) {
  __shared__ float scratch[32 * GR];
  __shared__ float f_s[GR + 1][kMaxSplits];
  __shared__ float L_s[GR + 1];
  const bool act = threadIdx.x < 2 * D;  // threads past 2D (wider blocks) only join the barriers
  const int ch = act ? threadIdx.x : 0;  // 0 .. 2D-1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int stride = 2 * D + 2;
  if (warp <= GR) {
    const int head = warp < GR ? g * GR + warp : q_origin + g;
    split_weights(ws + (int64_t)head * nsplit * stride, n_active, stride, f_s[warp], &L_s[warp], lane);
  }
  __syncthreads();
  // Σ_s f_j[s] · o_{j,s}[ch] for all GR+1 heads at once (their loads are independent).
  const float* hb[GR + 1];
  float acc[GR + 1];
#pragma unroll
  for (int j = 0; j <= GR; ++j) {
    hb[j] = ws + (int64_t)(j < GR ? g * GR + j : q_origin + g) * nsplit * stride + 2 + ch;
    acc[j] = 0.f;
  }
  int s = 0;
  for (; s + 2 <= n_active; s += 2) {
    float a0[GR + 1], a1[GR + 1];
#pragma unroll
    for (int j = 0; j <= GR; ++j) {
      a0[j] = __ldcg(hb[j] + s * stride);
      a1[j] = __ldcg(hb[j] + (s + 1) * stride);
    }
#pragma unroll
    for (int j = 0; j <= GR; ++j) acc[j] += f_s[j][s] * a0[j] + f_s[j][s + 1] * a1[j];
  }
  if (s < n_active) {
#pragma unroll
    for (int j = 0; j <= GR; ++j) acc[j] += f_s[j][s] * __ldcg(hb[j] + s * stride);
  }
  float val[GR + 1];
#pragma unroll
  for (int j = 0; j <= GR; ++j) val[j] = round_through<__half>(L_s[j] > 0.f ? acc[j] / L_s[j] : 0.f);
  float d[GR], ssq[GR];
#pragma unroll
  for (int j = 0; j < GR; ++j) {
    const int h_o = g * GR + j;
    const float l = lam[lam_mode == 0 ? 0 : (lam_mode == 1 ? g : h_o)];
    d[j] = val[j] - l * val[GR];
    ssq[j] = act ? d[j] * d[j] : 0.f;
  }
  block_sum<GR>(ssq, scratch);
  const float w = __half2float(subln_w[ch]);
#pragma unroll
  for (int j = 0; j < GR; ++j) {
    const float inv = rsqrtf(ssq[j] / (float)(2 * D) + eps);
    if (act) out[(int64_t)(g * GR + j) * 2 * D + ch] = __float2half_rn(d[j] * inv * w * out_scale);
  }
}

// Merge split partials of one vanilla group (NP pairs of signal head 2j, noise head 2j+1) and
// apply the differential combine of _forward_vanilla (model.py:553-557), rounding where the
// reference's fp16 arrays round: p = fp16(fp16(λ)·o2), d = fp16(o1 − p), y = fp16(rms_norm(d)·w),
// out = fp16(y·fp16(1 − λ_init)). Run by a CTA of 2D threads; out is (heads, 2D) of this group.
template <int D, int NP>
__device__ __forceinline__ void vanilla_merge_group(const float* __restrict__ ws, int nsplit, int n_active, int g,
                                                    const __half* __restrict__ subln_w,
                                                    const float* __restrict__ lam, float out_scale, float eps,
                                                    __half* __restrict__ out) {
  __shared__ float scratch[32 * NP];
  __shared__ float f_s[2 * NP][kMaxSplits];
  __shared__ float L_s[2 * NP];
  const bool act = threadIdx.x < 2 * D;  // threads past 2D (wider blocks) only join the barriers
  const int ch = act ? threadIdx.x : 0;  // 0 .. 2D-1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int stride = 2 * D + 2;
  if (warp < 2 * NP) {
    const int head = 2 * (g * NP + (warp >> 1)) + (warp & 1);
    split_weights(ws + (int64_t)head * nsplit * stride, n_active, stride, f_s[warp], &L_s[warp], lane);
  }
  __syncthreads();
  const float* hb[2 * NP];
  float acc[2 * NP];
#pragma unroll
  for (int j = 0; j < 2 * NP; ++j) {
    hb[j] = ws + (int64_t)(2 * (g * NP + (j >> 1)) + (j & 1)) * nsplit * stride + 2 + ch;
    acc[j] = 0.f;
  }
  for (int s = 0; s < n_active; ++s) {
    float a[2 * NP];
#pragma unroll
    for (int j = 0; j < 2 * NP; ++j) a[j] = __ldcg(hb[j] + s * stride);
#pragma unroll
    for (int j = 0; j < 2 * NP; ++j) acc[j] += f_s[j][s] * a[j];
  }
  const float lam16 = __half2float(__float2half_rn(lam[0]));
  float d[NP], ssq[NP];
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const float o1 = round_through<__half>(L_s[2 * j] > 0.f ? acc[2 * j] / L_s[2 * j] : 0.f);
    const float o2 = round_through<__half>(L_s[2 * j + 1] > 0.f ? acc[2 * j + 1] / L_s[2 * j + 1] : 0.f);
    d[j] = round_through<__half>(o1 - round_through<__half>(lam16 * o2));
    ssq[j] = act ? d[j] * d[j] : 0.f;
  }
  block_sum<NP>(ssq, scratch);
  const float w = __half2float(subln_w[ch]);
  const float os16 = __half2float(__float2half_rn(out_scale));
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const float inv = rsqrtf(ssq[j] / (float)(2 * D) + eps);
    const float y = round_through<__half>(d[j] * inv * w);
    if (act) out[(int64_t)(g * NP + j) * 2 * D + ch] = __float2half_rn(y * os16);
  }
}

template <int D, int GR>
__global__ void gda_combine_kernel(const float* __restrict__ ws, int nsplit, int kv_len_host,
                                   const int32_t* __restrict__ kv_len_dev, int q_origin,
                                   const __half* __restrict__ subln_w,
                                   const float* __restrict__ lam, int lam_mode, float out_scale,
                                   float eps, __half* __restrict__ out) {
  pdl_trigger();
  const int kv_len = kv_len_dev ? *kv_len_dev : kv_len_host;
  int p0, p1, n_active;
  split_range(kv_len, nsplit, 0, p0, p1, n_active);
  gda_merge_group<D, GR>(ws, nsplit, n_active, blockIdx.x, q_origin, subln_w, lam, lam_mode, out_scale, eps, out);
}

// ---- split partials merged through distributed shared memory ---------------------------------
//
// For short caches the splits of one group run as ONE thread-block cluster (grid.x = nsplit =
// cluster size). Each CTA stores its split's partial (m, l, o1|o2 per head) straight into the
// shared memory of the cluster's rank-0 CTA, arrives on the cluster barrier and exits — its SM
// is free for the next kernel at once; rank 0 waits on the barrier and merges the partials from
// its own shared memory: no global partials, fence, arrival counter or second pass through L2.
// The merge arithmetic and its summation order are gda_merge_group's, so both paths give the
// same bits. The cluster barrier is a hardware barrier over co-scheduled CTAs: no spinning.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Store to the shared-memory word at `p` (an address in this CTA's layout) of cluster rank `rank`.
__device__ __forceinline__ void st_dsmem(float* p, uint32_t rank, float v) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n"
               : "=r"(r)
               : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;\n" ::"r"(r), "f"(v) : "memory");
}

// gda_merge_group with the partials in this CTA's shared memory: all[s][h][2D + 2] holds split s
// (heads: GR origin heads, then the noise head).
template <int D, int GR>
__device__ __forceinline__ void gda_merge_group_smem(const float* all, int n_active, int g,
                                                     const __half* __restrict__ subln_w,
                                                     const float* __restrict__ lam, int lam_mode, float out_scale,
                                                     float eps, __half* __restrict__ out) {
  __shared__ float scratch[32 * GR];
  __shared__ float f_s[GR + 1][kMaxSplits];
  __shared__ float L_s[GR + 1];
  const bool act = threadIdx.x < 2 * D;
  const int ch = act ? threadIdx.x : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int stride = 2 * D + 2, split_stride = (GR + 1) * stride;
  if (warp <= GR) {  // split_weights over the splits held here (at most 32 of them)
    const float* base = all + warp * stride;
    const float m0 = lane < n_active ? base[lane * split_stride] : -INFINITY;
    const float m1 = -INFINITY;
    const float l0 = lane < n_active ? base[lane * split_stride + 1] : 0.f;
    const float l1 = 0.f;
    const float M = warp_max(fmaxf(m0, m1));
    const float f0 = (M != -INFINITY && m0 != -INFINITY) ? exp2f(m0 - M) : 0.f;
    const float f1 = 0.f;
    const float L = warp_sum(l0 * f0 + l1 * f1);
    f_s[warp][lane] = f0;
    f_s[warp][lane + 32] = f1;
    if (lane == 0) L_s[warp] = L;
  }
  __syncthreads();
  float acc[GR + 1];
#pragma unroll
  for (int j = 0; j <= GR; ++j) acc[j] = 0.f;
  int s = 0;
  for (; s + 2 <= n_active; s += 2) {
    float a0[GR + 1], a1[GR + 1];
#pragma unroll
    for (int j = 0; j <= GR; ++j) {
      a0[j] = all[s * split_stride + j * stride + 2 + ch];
      a1[j] = all[(s + 1) * split_stride + j * stride + 2 + ch];
    }
#pragma unroll
    for (int j = 0; j <= GR; ++j) acc[j] += f_s[j][s] * a0[j] + f_s[j][s + 1] * a1[j];
  }
  if (s < n_active) {
#pragma unroll
    for (int j = 0; j <= GR; ++j) acc[j] += f_s[j][s] * all[s * split_stride + j * stride + 2 + ch];
  }
  float val[GR + 1];
#pragma unroll
  for (int j = 0; j <= GR; ++j) val[j] = round_through<__half>(L_s[j] > 0.f ? acc[j] / L_s[j] : 0.f);
  float d[GR], ssq[GR];
#pragma unroll
  for (int j = 0; j < GR; ++j) {
    const int h_o = g * GR + j;
    const float l = lam[lam_mode == 0 ? 0 : (lam_mode == 1 ? g : h_o)];
    d[j] = val[j] - l * val[GR];
    ssq[j] = act ? d[j] * d[j] : 0.f;
  }
  block_sum<GR>(ssq, scratch);
  const float w = __half2float(subln_w[ch]);
#pragma unroll
  for (int j = 0; j < GR; ++j) {
    const float inv = rsqrtf(ssq[j] / (float)(2 * D) + eps);
    if (act) out[(int64_t)(g * GR + j) * 2 * D + ch] = __float2half_rn(d[j] * inv * w * out_scale);
  }
}

// ---- fused decode step: RoPE + 4-slot append + split-KV dual-V attention + GDA merge ----
//
// One launch per layer replaces rope_qkv_append, attn_split and gda_combine. Grid
// (nsplit, q_groups), 256 threads. Every CTA rotates the q heads of its group straight
// from the qkv row; the CTA whose position range holds `pos` first writes the new k/v
// row of its group (RoPE on k, quantized when the cache is) and then reads it back like
// any other row, so the attention sees exactly the stored values. Each CTA leaves its
// softmax partials in the workspace; the last CTA of a group to arrive (per-group
// counter at the head of the workspace, reset by that CTA) merges them and applies
// gda_post_split.
constexpr size_t kFusedCtlBytes = 256;  // per-group arrival counters (int32), zero between calls

struct FusedArgs {
  const __half* qkv;
  const float* inv_freq;
  int q_heads;   // q_origin + q_groups
  int q_origin;  // q_groups · gr
  int groups;    // q_groups = kv heads per slot
  motif_kv4_slots cache;
  const int32_t* pos_len;  // [pos, kv_len]
  float scale_log2;
  const __half* subln_w;
  const float* lam;
  int lam_mode;
  float out_scale;
  float eps;
  __half* out;
  float* ws;      // split partials
  int* counters;  // [groups]
};

// Query heads of a group: NA signal heads on k1 and NB noise heads on k2. GDA (PAIRED false):
// signal heads g·NA + j (origin-first), one noise head q_origin + g. Vanilla (PAIRED true,
// NB == NA): the stripes interleave, signal head 2·(g·NA + j) and its noise head right after.
template <int NA, int NB, bool PAIRED>
__device__ __forceinline__ int fused_head(int g, int h, int q_origin) {
  if (PAIRED) return 2 * (g * NA + (h < NA ? h : h - NA)) + (h < NA ? 0 : 1);
  return h < NA ? g * NA + h : q_origin + g;
}

template <int BITS, int NA, int NB, bool PAIRED, int PPW, int LPG, bool CLUSTER>
__global__ void __launch_bounds__(kAttnThreads) gda_fused_kernel(FusedArgs f) {
  constexpr int D = 128, CPL = D / 32, NH = NA + NB, half = D / 2;
  constexpr int kPosPerWarp = PPW, kRoundPositions = kAttnWarps * PPW;
  __shared__ float s_row[4][D];
  __shared__ float s_cs[half], s_sn[half];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int split = blockIdx.x, nsplit = gridDim.x;
  const int g = blockIdx.y;
  const int64_t cap = f.cache.capacity;
  // a device kv_len beyond the cache is clamped (never read past the slots)
  const int pos = f.pos_len[0], kv_len = max(0, min(f.pos_len[1], (int)cap));
  int p0, p1, n_active;
  split_range(kv_len, nsplit, split, p0, p1, n_active);
  if (n_active < 1) n_active = 1;  // kv_len 0: split 0 still merges (to zeros)
  // A split past the last active one has no rows. On the global path it leaves at once; in a
  // cluster it stays (every CTA takes part in the cluster barriers) with an empty range.
  if (!CLUSTER && split >= n_active) return;
  if (CLUSTER && split >= n_active) p0 = p1 = kv_len;
  const motif_kv4_slots& kv = f.cache;
  const int64_t row0 = (int64_t)g * cap;
  float ka[kPosPerWarp][CPL], kb[kPosPerWarp][CPL], x1[kPosPerWarp][CPL], x2[kPosPerWarp][CPL];
  auto load_round = [&](int base) {
#pragma unroll
    for (int u = 0; u < kPosPerWarp; ++u) {
      if (base + u < p1) {
        const int64_t r = row0 + base + u;
        load_kv<__half, D, BITS>(kv.data[0], kv.scales[0], kv.biases[0], r, lane, kv.group_size, ka[u]);
        load_kv<__half, D, BITS>(kv.data[1], kv.scales[1], kv.biases[1], r, lane, kv.group_size, kb[u]);
        load_kv<__half, D, BITS>(kv.data[2], kv.scales[2], kv.biases[2], r, lane, kv.group_size, x1[u]);
        load_kv<__half, D, BITS>(kv.data[3], kv.scales[3], kv.biases[3], r, lane, kv.group_size, x2[u]);
      }
    }
  };
  const bool append = pos >= 0 && pos < cap && ((pos >= p0 && pos < p1) || (split == 0 && pos >= kv_len));
  // The first round of this warp's rows does not depend on the RoPE work below, so it starts
  // now. In the appending CTA the warp whose first round holds row pos either loads it later
  // (quantized caches: the row is read back as stored) or, for fp16 rows, takes the new row
  // from shared memory after the append (the value it would read back, without the round trip).
  const int first = p0 + warp * kPosPerWarp;
  const bool holds_new = append && pos >= first && pos < first + kPosPerWarp && pos < p1;
  const bool defer = BITS != 16 && holds_new;
  if (!defer) load_round(first);
  // RoPE angles of this position, shared by every head of the CTA
  if (threadIdx.x < half) rope_angle(threadIdx.x, pos, f.inv_freq, s_cs[threadIdx.x], s_sn[threadIdx.x]);
  // Launched with programmatic serialization: everything above reads only data that
  // kernels before the previous one wrote (cache rows < pos, pos_len, inv_freq). The qkv
  // row comes from the previous kernel (the qkv projection): wait for it here.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  __syncthreads();

  // ---- rotated q of the group's GR origin heads and its noise head (its loads go out
  // before the append below, so the appending CTA waits for one round trip, not two) ----
  float q[NH][CPL];
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    const int head = fused_head<NA, NB, PAIRED>(g, h, f.q_origin);
    const __half* src = f.qkv + (int64_t)head * D;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = lane * CPL + j, k = c < half ? c : c - half;
      q[h][j] = __half2float(__float2half_rn(rope_rotate(src, c, half, s_cs[k], s_sn[k]))) * f.scale_log2;
    }
  }

  // ---- append the new row of this group (k1, k2, v1, v2 by warps 0..3) ----
  if (append) {
    if (warp < 4) {
      const int head = warp < 2 ? f.q_heads + 2 * g + warp : f.q_heads + 2 * f.groups + 2 * g + (warp - 2);
      const __half* src = f.qkv + (int64_t)head * D;
      const int64_t row = (int64_t)g * cap + pos;
      __half hv[CPL];
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int c = lane * CPL + j;
        const int k = c < half ? c : c - half;
        hv[j] = __float2half_rn(warp < 2 ? rope_rotate(src, c, half, s_cs[k], s_sn[k]) : __half2float(src[c]));
      }
      if constexpr (BITS == 16) {
        __half* dst = static_cast<__half*>(f.cache.data[warp]) + row * D + lane * CPL;
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          dst[j] = hv[j];
          s_row[warp][lane * CPL + j] = __half2float(hv[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < CPL; ++j) s_row[warp][lane * CPL + j] = __half2float(hv[j]);
        __syncwarp();
        // lanes 0 .. D/8-1 quantize 8 channels each (the others feed zeros to the shuffles)
        const bool act = lane < D / 8;
        float x8[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) x8[t] = act ? s_row[warp][lane * 8 + t] : 0.f;
        uint32_t words[2];
        float sc, bi;
        quant_group<LPG>(x8, BITS, words, sc, bi);
        if (act) {
          constexpr int EL = 32 / BITS;
          uint32_t* d = static_cast<uint32_t*>(f.cache.data[warp]) + row * (D / EL) + (lane * 8) / EL;
          d[0] = words[0];
          if constexpr (BITS == 8) d[1] = words[1];
          const int gs = f.cache.group_size;
          if (((lane * 8) % gs) == 0) {
            const int64_t gi = row * (D / gs) + (lane * 8) / gs;
            static_cast<__half*>(f.cache.scales[warp])[gi] = __float2half_rn(sc);
            static_cast<__half*>(f.cache.biases[warp])[gi] = __float2half_rn(bi);
          }
        }
      }
    }
    __syncthreads();  // the row is read back below (global writes ordered for the CTA)
  }

  float m[NH], l[NH], o1[NH][CPL], o2[NH][CPL];
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) o1[h][c] = o2[h][c] = 0.f;
  }
  if (defer) load_round(first);  // after the new row is written
  if (BITS == 16 && holds_new) {  // the new row, as stored, from shared memory
#pragma unroll
    for (int u = 0; u < kPosPerWarp; ++u) {
      if (first + u == pos) {
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          ka[u][j] = s_row[0][lane * CPL + j];
          kb[u][j] = s_row[1][lane * CPL + j];
          x1[u][j] = s_row[2][lane * CPL + j];
          x2[u][j] = s_row[3][lane * CPL + j];
        }
      }
    }
  }
  for (int base = p0 + warp * kPosPerWarp; base < p1; base += kRoundPositions) {
    if (base != p0 + warp * kPosPerWarp) load_round(base);
#pragma unroll
    for (int u = 0; u < kPosPerWarp; ++u) {
      if (base + u >= p1) break;
      float s[NH];
#pragma unroll
      for (int h = 0; h < NH; ++h) {  // signal heads score on k1, noise heads on k2
        float t = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) t += q[h][c] * (h < NA ? ka[u][c] : kb[u][c]);
        s[h] = t;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int h = 0; h < NH; ++h) s[h] += __shfl_xor_sync(0xffffffffu, s[h], o);
      }
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const float mn = fmaxf(m[h], s[h]);
        const float fac = exp2f(m[h] - mn);
        const float e = exp2f(s[h] - mn);
        m[h] = mn;
        l[h] = l[h] * fac + e;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          o1[h][c] = o1[h][c] * fac + e * x1[u][c];
          o2[h][c] = o2[h][c] * fac + e * x2[u][c];
        }
      }
    }
  }

  // The next kernel (the o projection) may start streaming its weights now: this CTA's
  // cache reads are done, so they no longer compete with it.
  pdl_trigger();
  // ---- merge the warps' partial softmax states, write this split's partials ----
  extern __shared__ float smem[];
  float* sm_ml = smem;                       // [warp][h][2]
  float* sm_o = smem + kAttnWarps * NH * 2;  // [warp][h][2D]
  float* part_s = sm_o + kAttnWarps * NH * 2 * D;  // cluster path, rank 0: [split][h][2D + 2]
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    if (lane == 0) {
      sm_ml[(warp * NH + h) * 2 + 0] = m[h];
      sm_ml[(warp * NH + h) * 2 + 1] = l[h];
    }
    float* dst = sm_o + (int64_t)(warp * NH + h) * 2 * D + lane * CPL;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      dst[c] = o1[h][c];
      dst[D + c] = o2[h][c];
    }
  }
  // Per head: the running maximum over the warps and each warp's rescale factor, once (the
  // channel loop below then needs one factor load per warp); same arithmetic and order as
  // rescaling in the channel loop itself.
  __shared__ float s_fw[kAttnWarps][NH];
  __shared__ float s_M[NH], s_L[NH];
  __shared__ unsigned s_live[NH];
  __syncthreads();  // every warp's state is in shared memory
  if (threadIdx.x < NH) {
    const int h = threadIdx.x;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_ml[(w * NH + h) * 2]);
    float L = 0.f;
    unsigned live = 0;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float mw = sm_ml[(w * NH + h) * 2];
        if (mw == -INFINITY) continue;
        const float fw = exp2f(mw - M);
        s_fw[w][h] = fw;
        live |= 1u << w;
        L += sm_ml[(w * NH + h) * 2 + 1] * fw;
      }
    }
    s_M[h] = M;
    s_L[h] = L;
    s_live[h] = live;
  }
  __syncthreads();
  for (int it = threadIdx.x; it < NH * 2 * D; it += kAttnThreads) {
    const int h = it / (2 * D);
    const int ch = it - h * 2 * D;
    const float M = s_M[h], L = s_L[h];
    const unsigned live = s_live[h];
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w)
      if (live & (1u << w)) O += sm_o[(int64_t)(w * NH + h) * 2 * D + ch] * s_fw[w][h];
    if constexpr (CLUSTER) {  // into rank 0's shared memory, slot `split`
      float* p = part_s + ((int64_t)split * NH + h) * (2 * D + 2);
      st_dsmem(p + 2 + ch, 0, O);
      if (ch == 0) {
        st_dsmem(p, 0, M);
        st_dsmem(p + 1, 0, L);
      }
    } else {
      const int hh = fused_head<NA, NB, PAIRED>(g, h, f.q_origin);
      float* p = f.ws + ((int64_t)hh * nsplit + split) * (2 * D + 2);
      p[2 + ch] = O;
      if (ch == 0) {
        p[0] = M;
        p[1] = L;
      }
    }
  }
  if constexpr (CLUSTER) {
    static_assert(!PAIRED && NB == 1, "the cluster merge is built for the GDA head layout");
    cluster_arrive_release();  // this split's partial is in rank 0's shared memory
    if (cluster_rank() != 0) return;
    cluster_wait_acquire();  // every split's partial has arrived
    gda_merge_group_smem<D, NA>(part_s, n_active, g, f.subln_w, f.lam, f.lam_mode, f.out_scale, f.eps, f.out);
    return;
  }

  // ---- the last CTA of the group merges ----
  __threadfence();  // release this CTA's partials before counting in
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(f.counters + g, 1) == n_active - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // acquire the other CTAs' partials
  if constexpr (PAIRED)
    vanilla_merge_group<D, NA>(f.ws, nsplit, n_active, g, f.subln_w, f.lam, f.out_scale, f.eps, f.out);
  else
    gda_merge_group<D, NA>(f.ws, nsplit, n_active, g, f.q_origin, f.subln_w, f.lam, f.lam_mode, f.out_scale, f.eps,
                           f.out);
  if (threadIdx.x == 0) f.counters[g] = 0;  // ready for the next launch
}

// ---- long-context decode step on the tensor cores ------------------------------------------
//
// Same contract as gda_fused_kernel (RoPE + append of the new row, split-KV attention over the
// cache, last-CTA merge with the differential combine), for caches long enough that the
// per-position CUDA-core work limits gda_fused_kernel. Cache positions are the MMA's M
// dimension: per 128-position tile
//   S1ᵀ = K1·Q_sigᵀ and S2ᵀ = K2·Q_noiseᵀ      (M 128 positions, N 16 padded heads, K 128)
//   O1ᵀ += V1ᵀ·Pᵀ and O2ᵀ += V2ᵀ·Pᵀ            (M 128 channels, N 16 heads, K 128 positions;
//                                               V read MN-major: the cache rows as stored)
// with S and O in tensor memory. Warps 2..5 (one thread per position, then per channel) run
// the online softmax — per-head maxima through shuffles and a barrier, the running maximum
// re-based only when it grows by more than 2^8 (O's columns rescaled in tensor memory), P
// written as fp16 — and store the split's partial (m, l, O) in the layout the merge reads.
//   fp16 cache (BITS 16): warp 0 streams (k1, k2) and (v1, v2) tile pairs with TMA straight
//     into a three-entry ring of 64 KB operand tiles (128-byte swizzle); warp 1 issues QK one
//     tile ahead of PV.
//   q4 cache (BITS 4, group 64): warp 0 streams the packed rows (codes, scales, biases of the
//     four slots: 36 KB a tile) into a two-entry ring; warps 6..13 dequantize them (1024 + q
//     exponent trick, one fused multiply-add with scale and bias) into two fp16 operand
//     entries (K, V) in the same swizzled layout; warp 1 issues PV(j) then QK(j+1).
// Splits start on multiples of 128 positions (the packed-scale view needs 4-row alignment).
constexpr int kLT = 128;  // cache positions per tile
constexpr int kLErrSlot = 63;  // control word set to 1 when a wait timed out

template <int BITS>
struct LongCfg;
template <>
struct LongCfg<16> {
  static constexpr int kThreads = 256;
  static constexpr int kRing = 3;                 // 64 KB operand entries
  static constexpr int kOffQ = kRing * 65536;     // Q_sig, Q_noise: 2 × 4 KB
  static constexpr int kOffP = kOffQ + 8192;      // Pᵀ: 2 × 4 KB
  static constexpr int kOffRed = kOffP + 8192;    // softmax scratch (768 B)
  static constexpr int kOffRow = kOffRed + 1024;  // append scratch (unused for fp16)
  static constexpr int kOffBar = kOffRow;
  static constexpr int kBars = 2 * kRing + 7;     // full[3], free[3], s_full[2], p_full[2], o_bar[2], drain
};
template <>
struct LongCfg<4> {
  static constexpr int kThreads = 448;
  static constexpr int kPacked = 36864;            // codes 4 × 8 KB, scales 4 × 512 B, biases 4 × 512 B
  static constexpr int kOffPk = 131072;            // after the two 64 KB operand entries
  static constexpr int kOffQ = kOffPk + 2 * kPacked;
  static constexpr int kOffP = kOffQ + 8192;
  static constexpr int kOffRed = kOffP + 8192;
  static constexpr int kOffRow = kOffPk + kPacked;  // append scratch aliases packed entry 1 (free then)
  static constexpr int kOffBar = kOffRed + 1024;
  static constexpr int kBars = 15;  // ofull[2], ofree[2], pfull[2], pfree[2], s_full[2], p_full[2], o_bar[2], drain
};
template <int BITS>
constexpr int long_smem() {
  return LongCfg<BITS>::kOffBar + LongCfg<BITS>::kBars * 8 + 16 + 1024;
}

struct LongMaps {
  CUtensorMap slot[4];  // fp16: rows × 256 B, box 128 B × 128, swizzled; q4: codes rows × 64 B, box 64 B × 128
  CUtensorMap sc[4];    // q4 scales / biases as 16-byte lines (4 rows each), box 16 B × 32
  CUtensorMap bi[4];
};

// Byte offset of element (row, col) in a K-major tile of 16 rows × 128 fp16 (two 64-column
// chunks of 16 rows × 128 B, 128-byte swizzle).
__device__ __forceinline__ uint32_t kmaj16_off(int row, int col) {
  return (uint32_t)((col >> 6) * 2048 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

// Split ranges of the tensor-core step: chunks rounded up to whole tiles.
__device__ __forceinline__ void long_split_range(int kv_len, int nsplit, int split, int& p0, int& p1, int& n_active) {
  int chunk = (kv_len + nsplit - 1) / nsplit;
  chunk = ((chunk + kLT - 1) / kLT) * kLT;
  if (chunk < kLT) chunk = kLT;
  n_active = (kv_len + chunk - 1) / chunk;
  p0 = split * chunk;
  p1 = min(kv_len, p0 + chunk);
}

__device__ __forceinline__ uint32_t dq_half2(uint32_t p, __half2 s2, __half2 b2) {
  const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));
  __half2 h = *reinterpret_cast<__half2*>(&p);
  h = __hfma2(__hsub2(h, k1024), s2, b2);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Eight nibbles (element e at bits 4e..4e+3) -> eight fp16 values in element order.
__device__ __forceinline__ uint4 dq_word(uint32_t w, __half2 s2, __half2 b2) {
  const uint32_t t0 = (w & 0x000F000Fu) | 0x64006400u;
  const uint32_t t1 = ((w >> 4) & 0x000F000Fu) | 0x64006400u;
  const uint32_t t2 = ((w >> 8) & 0x000F000Fu) | 0x64006400u;
  const uint32_t t3 = ((w >> 12) & 0x000F000Fu) | 0x64006400u;
  uint4 o;
  o.x = dq_half2(__byte_perm(t0, t1, 0x5410), s2, b2);
  o.y = dq_half2(__byte_perm(t2, t3, 0x5410), s2, b2);
  o.z = dq_half2(__byte_perm(t0, t1, 0x7632), s2, b2);
  o.w = dq_half2(__byte_perm(t2, t3, 0x7632), s2, b2);
  return o;
}

template <int NA, int NB, bool PAIRED, int BITS>
__global__ void __launch_bounds__(LongCfg<BITS>::kThreads, 1)
    gda_long_kernel(FusedArgs f, const __grid_constant__ LongMaps tm) {
  using C = LongCfg<BITS>;
  constexpr int D = 128, NH = NA + NB, half = D / 2;
  constexpr bool Q4 = BITS == 4;
  static_assert(NA <= 16 && NB <= 16, "heads per group");
  __shared__ float s_cs[half], s_sn[half];
  __shared__ int s_last;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = tc::smem_addr(smem);
  const uint32_t bar = sb + C::kOffBar;
  // barrier map: fp16 full[e] 0..2, free[e] 3..5; q4 ofull[2] 0..1, ofree[2] 2..3, pfull[2] 4..5, pfree[2] 6..7
  constexpr int kS = Q4 ? 8 : 6;
  auto s_full = [&](int b) { return bar + 8u * (kS + b); };
  auto p_full = [&](int b) { return bar + 8u * (kS + 2 + b); };
  // PV(j) completes phase j / 2 of o_bar(j mod 2): a wait for PV(k) can only have PV(k+2) (same
  // barrier, next phase) behind it, which needs P(k+2) from the waiting thread itself.
  auto o_bar = [&](int b) { return bar + 8u * (kS + 4 + b); };
  const uint32_t drain = bar + 8u * (kS + 6);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + C::kOffRed);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int split = blockIdx.x, nsplit = gridDim.x, g = blockIdx.y;
  const int64_t cap = f.cache.capacity;
  // every read below may depend on the previous kernel (the qkv projection)
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  const int pos = f.pos_len[0], kv_len = max(0, min(f.pos_len[1], (int)cap));
  int p0, p1, n_active;
  long_split_range(kv_len, nsplit, split, p0, p1, n_active);
  if (n_active < 1) n_active = 1;
  if (split >= n_active) return;
  const bool append = pos >= 0 && pos < cap && ((pos >= p0 && pos < p1) || (split == 0 && pos >= kv_len));
  const int nt = p1 > p0 ? (p1 - p0 + kLT - 1) / kLT : 0;

  if (threadIdx.x < half) rope_angle(threadIdx.x, pos, f.inv_freq, s_cs[threadIdx.x], s_sn[threadIdx.x]);
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kBars; ++i) {
      int cnt = 1;
      if (i == kS + 2 || i == kS + 3) cnt = 4;                     // p_full: the four softmax warps
      if (Q4 && (i <= 1 || i == 6 || i == 7)) cnt = 8;             // ofull, pfree: the dequant warps
      tc::mbar_init(bar + 8u * i, cnt);
    }
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_addr(tmem_slot), 128);  // S: 2 × 32 columns, O1/O2: 2 × 16
    tc::tmem_relinquish();
  }
  // zero the Q and Pᵀ tiles (rows past NH stay zero: padded heads)
  for (int i = threadIdx.x; i < 16384 / 16; i += C::kThreads)
    reinterpret_cast<uint4*>(smem + C::kOffQ)[i] = make_uint4(0, 0, 0, 0);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- the new row (k1, k2 with RoPE, v1, v2) of this group, by warps 0..3 ----
  if (append && warp < 4) {
    const int head = warp < 2 ? f.q_heads + 2 * g + warp : f.q_heads + 2 * f.groups + 2 * g + (warp - 2);
    const __half* src = f.qkv + (int64_t)head * D;
    const int64_t row = (int64_t)g * cap + pos;
    __half hv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = lane * 4 + j, k = c < half ? c : c - half;
      hv[j] = __float2half_rn(warp < 2 ? rope_rotate(src, c, half, s_cs[k], s_sn[k]) : __half2float(src[c]));
    }
    if constexpr (!Q4) {
      __half* dst = static_cast<__half*>(f.cache.data[warp]) + row * D + lane * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = hv[j];
    } else {
      float* s_row = reinterpret_cast<float*>(smem + C::kOffRow) + warp * D;
#pragma unroll
      for (int j = 0; j < 4; ++j) s_row[lane * 4 + j] = __half2float(hv[j]);
      __syncwarp();
      const bool act = lane < D / 8;
      float x8[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) x8[t] = act ? s_row[lane * 8 + t] : 0.f;
      uint32_t words[2];
      float scv, biv;
      quant_group<8>(x8, 4, words, scv, biv);
      if (act) {
        static_cast<uint32_t*>(f.cache.data[warp])[row * (D / 8) + lane] = words[0];
        if ((lane * 8) % 64 == 0) {
          const int64_t gi = row * (D / 64) + (lane * 8) / 64;
          static_cast<__half*>(f.cache.scales[warp])[gi] = __float2half_rn(scv);
          static_cast<__half*>(f.cache.biases[warp])[gi] = __float2half_rn(biv);
        }
      }
    }
    asm volatile("fence.proxy.async.global;\n" ::: "memory");  // the TMA loads below read this row
  }
  // ---- rotated q of the group's heads, fp16, into the K-major Q tiles ----
  for (int i = threadIdx.x; i < NH * D; i += C::kThreads) {
    const int h = i / D, c = i - h * D, k = c < half ? c : c - half;
    const __half* src = f.qkv + (int64_t)fused_head<NA, NB, PAIRED>(g, h, f.q_origin) * D;
    const __half v = __float2half_rn(rope_rotate(src, c, half, s_cs[k], s_sn[k]));
    const int tile = h < NA ? 0 : 1, row = h < NA ? h : h - NA;
    *reinterpret_cast<__half*>(smem + C::kOffQ + tile * 4096 + kmaj16_off(row, c)) = v;
  }
  tc::fence_proxy_async_smem();
  __syncthreads();

  const int64_t row0 = (int64_t)g * cap + p0;
  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer ----
      if constexpr (!Q4) {  // (k1,k2) then (v1,v2) operand tiles per tile
        auto full = [&](int e) { return bar + 8u * e; };
        auto freeb = [&](int e) { return bar + 8u * (C::kRing + e); };
        int issued = 0;
        for (int u = 0; u < 2 * nt; ++u) {
          const int e = u % C::kRing, r = u / C::kRing;
          if (u >= C::kRing && !tc::mbar_wait(freeb(e), (r - 1) & 1)) { *abort_flag = 1; break; }
          if (*abort_flag) break;
          const int jj = u >> 1, sl = (u & 1) * 2;
          const int row = (int)(row0 + jj * kLT);
          const uint32_t dst = sb + e * 65536;
          tc::mbar_expect_tx(full(e), 65536);
          tc::tma_load_2d(dst, &tm.slot[sl], 0, row, full(e));
          tc::tma_load_2d(dst + 16384, &tm.slot[sl], 128, row, full(e));
          tc::tma_load_2d(dst + 32768, &tm.slot[sl + 1], 0, row, full(e));
          tc::tma_load_2d(dst + 49152, &tm.slot[sl + 1], 128, row, full(e));
          issued = u + 1;
        }
        for (int u = issued > C::kRing ? issued - C::kRing : 0; u < issued; ++u)
          if (!tc::mbar_wait(full(u % C::kRing), (u / C::kRing) & 1)) *abort_flag = 1;
      } else {  // packed rows of the four slots per tile
        auto pfull = [&](int e) { return bar + 8u * (4 + e); };
        auto pfree = [&](int e) { return bar + 8u * (6 + e); };
        int issued = 0;
        for (int jj = 0; jj < nt; ++jj) {
          const int e = jj & 1;
          if (jj >= 2 && !tc::mbar_wait(pfree(e), ((jj >> 1) - 1) & 1)) { *abort_flag = 1; break; }
          if (*abort_flag) break;
          const int row = (int)(row0 + jj * kLT);
          const uint32_t dst = sb + C::kOffPk + e * C::kPacked;
          tc::mbar_expect_tx(pfull(e), C::kPacked);
#pragma unroll
          for (int sl = 0; sl < 4; ++sl) {
            tc::tma_load_2d(dst + sl * 8192, &tm.slot[sl], 0, row, pfull(e));
            tc::tma_load_2d(dst + 32768 + sl * 512, &tm.sc[sl], 0, row / 4, pfull(e));
            tc::tma_load_2d(dst + 34816 + sl * 512, &tm.bi[sl], 0, row / 4, pfull(e));
          }
          issued = jj + 1;
        }
        for (int jj = issued > 2 ? issued - 2 : 0; jj < issued; ++jj)
          if (!tc::mbar_wait(pfull(jj & 1), (jj >> 1) & 1)) *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer ----
      constexpr uint32_t idesc_qk = tc::idesc_f16_f32(kLT, 16);
      constexpr uint32_t idesc_pv = tc::idesc_f16_f32(kLT, 16, false, true);
      const uint32_t qs = sb + C::kOffQ, qn = sb + C::kOffQ + 4096;
      // operand entry holding K(j) / V(j), the barrier saying it is ready, and the one to free
      auto k_entry = [&](int jj) { return Q4 ? 0 : (2 * jj) % 3; };
      auto v_entry = [&](int jj) { return Q4 ? 1 : (2 * jj + 1) % 3; };
      auto ready = [&](int e, int use) -> bool {  // `use`: how many times this entry was filled before
        return tc::mbar_wait(bar + 8u * e, use & 1);
      };
      auto freebar = [&](int e) { return bar + 8u * ((Q4 ? 2 : 3) + e); };
      auto issue_qk = [&](int jj) -> bool {
        const int e = k_entry(jj);
        if (!ready(e, Q4 ? jj : (2 * jj) / 3)) return false;
        tc::tc_fence_after();
        const uint32_t kb = sb + e * 65536;
        const uint32_t col = (jj & 1) * 32;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ko = (kk >> 2) * 16384 + (kk & 3) * 32, qo = (kk >> 2) * 2048 + (kk & 3) * 32;
          tc::mma_f16(tmem + col, tc::desc_kmajor_sw128(kb + ko), tc::desc_kmajor_sw128(qs + qo), idesc_qk, kk > 0);
          tc::mma_f16(tmem + col + 16, tc::desc_kmajor_sw128(kb + 32768 + ko), tc::desc_kmajor_sw128(qn + qo),
                      idesc_qk, kk > 0);
        }
        tc::mma_commit(s_full(jj & 1));
        tc::mma_commit(freebar(e));
        return true;
      };
      auto issue_pv = [&](int jj) -> bool {
        const int e = v_entry(jj);
        if (!tc::mbar_wait(p_full(jj & 1), (jj >> 1) & 1) || !ready(e, Q4 ? jj : (2 * jj + 1) / 3)) return false;
        tc::tc_fence_after();
        const uint32_t vb = sb + e * 65536, pb = sb + C::kOffP + (jj & 1) * 4096;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t bdesc = tc::desc_kmajor_sw128(pb + (kk >> 2) * 2048 + (kk & 3) * 32);
          tc::mma_f16(tmem + 64, tc::desc_mnmajor_sw128(vb + kk * 2048, 16384, 1024), bdesc, idesc_pv,
                      (jj | kk) != 0);
          tc::mma_f16(tmem + 80, tc::desc_mnmajor_sw128(vb + 32768 + kk * 2048, 16384, 1024), bdesc, idesc_pv,
                      (jj | kk) != 0);
        }
        tc::mma_commit(o_bar(jj & 1));
        tc::mma_commit(freebar(e));
        return true;
      };
      bool ok = nt == 0 || issue_qk(0);
      for (int jj = 0; ok && jj < nt; ++jj) {
        if (*abort_flag) { ok = false; break; }
        if constexpr (!Q4) {  // QK one tile ahead: its K tile is already in the ring
          if (jj + 1 < nt && !issue_qk(jj + 1)) { ok = false; break; }
          if (!issue_pv(jj)) { ok = false; break; }
        } else {  // K(j+1) is dequantized into the one K entry after QK(j): PV(j) first
          if (!issue_pv(jj)) { ok = false; break; }
          if (jj + 1 < nt && !issue_qk(jj + 1)) { ok = false; break; }
        }
      }
      if (!ok) *abort_flag = 1;
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0)) *abort_flag = 1;
    }
    __syncwarp();
  } else if (warp < 6) {  // ---- softmax: thread = position of the tile, later = channel ----
    const int sw = warp - 2, q = warp & 3, r = q * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    float m_ref[NH], L[NH];
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      m_ref[h] = -INFINITY;
      L[h] = 0.f;
    }
    int o_seen = 0;
    bool alive = true;
    auto observe = [&](int upto) -> bool {  // PV(0 .. upto-1) complete, in order
      while (o_seen < upto) {
        if (!tc::mbar_wait(o_bar(o_seen & 1), (o_seen >> 1) & 1)) return false;
        ++o_seen;
      }
      return true;
    };
    for (int j = 0; j < nt; ++j) {
      const bool got = tc::mbar_wait(s_full(j & 1), (j >> 1) & 1);
      tc::tc_fence_after();
      uint32_t s1[16], s2[16];
      tc::tmem_ld16(trow + (j & 1) * 32, s1);
      tc::tmem_ld16(trow + (j & 1) * 32 + 16, s2);
      tc::tmem_ld_wait();
      const bool valid = p0 + j * kLT + r < p1;
      float x[NH], mt[NH];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        x[h] = valid ? __uint_as_float(h < NA ? s1[h] : s2[h - NA]) * f.scale_log2 : -INFINITY;
        mt[h] = warp_max(x[h]);
      }
      float* rb = red + (j & 1) * 64;
      if (lane == 0)
#pragma unroll
        for (int h = 0; h < NH; ++h) rb[sw * 16 + h] = mt[h];
      // the four warps leave together when a wait gave up anywhere
      if (tc::named_sync_or(1, 128, !got || *abort_flag)) {
        *abort_flag = 1;
        alive = false;
        break;
      }
      bool any_need = false;
      float factor[NH];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const float m = fmaxf(fmaxf(rb[h], rb[16 + h]), fmaxf(rb[32 + h], rb[48 + h]));
        factor[h] = 1.f;
        if (m > m_ref[h] + 8.f) {
          factor[h] = exp2f(m_ref[h] - m);  // 0 while nothing was accumulated (m_ref = -inf)
          m_ref[h] = m;
          any_need = true;
        }
        L[h] *= factor[h];
      }
      __half pv[NH];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        pv[h] = __float2half_rn(x[h] == -INFINITY ? 0.f : exp2f(x[h] - m_ref[h]));
        L[h] += __half2float(pv[h]);
      }
      // Pᵀ buffer (j mod 2) was last read by PV(j-2); a rescale of O also needs PV(j-1) finished.
      // PV(j-1) otherwise keeps running while this tile's softmax proceeds.
      bool okw = observe(j - 1);
      if (okw && any_need && j > 0) {
        okw = observe(j);
        if (__all_sync(0xffffffffu, okw)) {
          tc::tc_fence_after();
#pragma unroll
          for (int oc = 0; oc < 2; ++oc) {
            uint32_t ov[16];
            tc::tmem_ld16(trow + 64 + oc * 16, ov);
            tc::tmem_ld_wait();
#pragma unroll
            for (int h = 0; h < NH; ++h) ov[h] = __float_as_uint(__uint_as_float(ov[h]) * factor[h]);
            tc::tmem_st16(trow + 64 + oc * 16, ov);
          }
          tc::tmem_st_wait();
        }
      }
      if (!okw) *abort_flag = 1;  // caught by the next tile's barrier (or the final wait)
      uint8_t* pt = smem + C::kOffP + (j & 1) * 4096;
#pragma unroll
      for (int h = 0; h < NH; ++h) *reinterpret_cast<__half*>(pt + kmaj16_off(h, r)) = pv[h];
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(p_full(j & 1));
    }
    // ---- the split's partial: O columns per channel r, m and l per head ----
    const bool fin = alive && __all_sync(0xffffffffu, observe(nt));
    if (!fin) *abort_flag = 1;
    tc::tc_fence_after();
    uint32_t o1[16], o2[16];
    tc::tmem_ld16(trow + 64, o1);
    tc::tmem_ld16(trow + 80, o2);
    tc::tmem_ld_wait();
    float* lred = red + 128;
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      const float t = warp_sum(L[h]);
      if (lane == 0) lred[sw * 16 + h] = t;
    }
    tc::named_sync(1, 128);
    constexpr int stride = 2 * D + 2;
    const bool any = nt > 0 && fin;
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      float* base = f.ws + ((int64_t)fused_head<NA, NB, PAIRED>(g, h, f.q_origin) * nsplit + split) * stride;
      base[2 + r] = any ? __uint_as_float(o1[h]) : 0.f;
      base[2 + D + r] = any ? __uint_as_float(o2[h]) : 0.f;
      if (r == 0) {
        base[0] = any ? m_ref[h] : -INFINITY;
        base[1] = any ? (lred[h] + lred[16 + h]) + (lred[32 + h] + lred[48 + h]) : 0.f;
      }
    }
  } else if constexpr (Q4) {  // ---- dequantize packed tiles into the operand entries ----
    const int t = threadIdx.x - 192;  // 0..255: slot (t >> 7) of the pair, row (t & 127)
    const int sp = t >> 7, p = t & 127;
    auto ofull = [&](int e) { return bar + 8u * e; };
    auto ofree = [&](int e) { return bar + 8u * (2 + e); };
    auto pfull = [&](int e) { return bar + 8u * (4 + e); };
    auto pfree = [&](int e) { return bar + 8u * (6 + e); };
    for (int u = 0; u < 2 * nt; ++u) {
      const int jj = u >> 1, part = u & 1, e = jj & 1;
      bool okd = true;
      if (part == 0) okd = tc::mbar_wait(pfull(e), (jj >> 1) & 1);
      if (okd && jj > 0) okd = tc::mbar_wait(ofree(part), (jj - 1) & 1);  // MMA done with this entry's last use
      if (__any_sync(0xffffffffu, !okd || *abort_flag)) {
        *abort_flag = 1;
        break;
      }
      const int sl = part * 2 + sp;
      const uint8_t* pk = smem + C::kOffPk + e * C::kPacked;
      const uint4* codes = reinterpret_cast<const uint4*>(pk + sl * 8192 + p * 64);
      const __half2 sc2 = *reinterpret_cast<const __half2*>(pk + 32768 + sl * 512 + p * 4);
      const __half2 bi2 = *reinterpret_cast<const __half2*>(pk + 34816 + sl * 512 + p * 4);
      uint8_t* dst = smem + part * 65536 + sp * 32768 + p * 128;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint4 cw = codes[v];
        const uint32_t wv[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int w = v * 4 + k;  // channels 8w .. 8w+7, group w >> 3
          const __half2 s2 = __half2half2(w < 8 ? __low2half(sc2) : __high2half(sc2));
          const __half2 b2 = __half2half2(w < 8 ? __low2half(bi2) : __high2half(bi2));
          *reinterpret_cast<uint4*>(dst + (w >> 3) * 16384 + (((w & 7) ^ (p & 7)) << 4)) = dq_word(wv[k], s2, b2);
        }
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(ofull(part));
        if (part == 1) tc::mbar_arrive(pfree(e));
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 128);
  }
  pdl_trigger();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(f.counters + kLErrSlot, 1);
  // ---- the last CTA of the group merges the splits ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(f.counters + g, 1) == n_active - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if constexpr (PAIRED)
    vanilla_merge_group<D, NA>(f.ws, nsplit, n_active, g, f.subln_w, f.lam, f.out_scale, f.eps, f.out);
  else
    gda_merge_group<D, NA>(f.ws, nsplit, n_active, g, f.q_origin, f.subln_w, f.lam, f.lam_mode, f.out_scale, f.eps,
                           f.out);
  if (threadIdx.x == 0) f.counters[g] = 0;
}

template <typename T, int D, int BITS, int MAXA, int NB>
int launch_split(const AttnArgs& a, int nsplit, int batch, cudaStream_t st) {
  constexpr int NH = MAXA + NB;
  const size_t smem = sizeof(float) * (size_t)kAttnWarps * NH * (2 + 2 * D);
  auto kern = attn_split_kernel<T, D, BITS, MAXA, NB>;
  static bool configured = false;  // one attribute call per instantiation
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "attention: smem attribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  dim3 grid(nsplit, batch * a.h_kv);
  kern<<<grid, kAttnThreads, smem, st>>>(a);
  return check_launch("attention split");
}

template <typename T, int D, int BITS>
int dispatch_generic(AttnArgs& a, int G, int nsplit, int batch, cudaStream_t st) {
  if (G == 1) return launch_split<T, D, BITS, 1, 0>(a, nsplit, batch, st);
  if (G <= 4) return launch_split<T, D, BITS, 4, 0>(a, nsplit, batch, st);
  return launch_split<T, D, BITS, 8, 0>(a, nsplit, batch, st);
}

int choose_splits(int64_t groups, int64_t len_bound, int64_t max_splits) {
  // Aim for ~2 CTAs per SM across 148 SMs, never below kMinChunk positions per split.
  int64_t want = ceil_div(296, groups < 1 ? 1 : groups);
  int64_t by_len = ceil_div(len_bound < 1 ? 1 : len_bound, kMinChunk);
  int64_t n = want < by_len ? want : by_len;
  if (n > max_splits) n = max_splits;
  if (n > kMaxSplits) n = kMaxSplits;
  if (n < 1) n = 1;
  return (int)n;
}

size_t partial_bytes(int64_t rows, int64_t D, int64_t nsplit) {
  return sizeof(float) * (size_t)rows * (size_t)nsplit * (size_t)(2 * D + 2);
}

template <typename T>
int run_generic(int bits, AttnArgs& a, int64_t batch, int64_t h_q, int64_t h_kv, int64_t cap,
                int64_t D, int64_t kv_len, void* workspace, size_t ws_bytes, cudaStream_t st) {
  const int G = (int)(h_q / h_kv);
  const int64_t len_bound = a.kv_len_dev ? cap : kv_len;
  const int64_t max_splits_ws = ws_bytes / partial_bytes(batch * h_q, D, 1);
  int nsplit = choose_splits(batch * h_kv, len_bound, max_splits_ws);
  if (!workspace || ws_bytes == 0) nsplit = 1;
  a.ws = static_cast<float*>(workspace);
  a.force_partials = 0;
  int rc;
#define MOTIF_RUN_D(DD)                                                                  \
  if (bits == 16) rc = dispatch_generic<T, DD, 16>(a, G, nsplit, (int)batch, st);        \
  else if (bits == 4) rc = dispatch_generic<T, DD, 4>(a, G, nsplit, (int)batch, st);     \
  else rc = dispatch_generic<T, DD, 8>(a, G, nsplit, (int)batch, st);
  if (D == 64) {
    MOTIF_RUN_D(64)
  } else {
    MOTIF_RUN_D(128)
  }
#undef MOTIF_RUN_D
  if (rc != MOTIF_OK || nsplit == 1) return rc;
  if (D == 64)
    attn_combine_kernel<T, 64><<<batch * h_q, 128, 0, st>>>(a.ws, nsplit, (int)kv_len, a.kv_len_dev, static_cast<T*>(a.y));
  else
    attn_combine_kernel<T, 128><<<batch * h_q, 256, 0, st>>>(a.ws, nsplit, (int)kv_len, a.kv_len_dev, static_cast<T*>(a.y));
  return check_launch("attention combine");
}

int check_common(int64_t batch, int64_t h_q, int64_t h_kv, int64_t cap, int64_t D, int64_t kv_len,
                 const int32_t* kv_len_dev) {
  MOTIF_REQUIRE(batch > 0 && h_q > 0 && h_kv > 0 && cap >= 0, MOTIF_ERR_BAD_SHAPE,
                "sdpa_dual_v: bad shape B=%lld H_q=%lld H_kv=%lld cap=%lld", (long long)batch,
                (long long)h_q, (long long)h_kv, (long long)cap);
  MOTIF_REQUIRE(D % 32 == 0, MOTIF_ERR_BAD_CONTRACT, "sdpa_dual_v: D=%lld must be a multiple of 32", (long long)D);
  MOTIF_REQUIRE(D == 64 || D == 128, MOTIF_ERR_BAD_CONTRACT,
                "sdpa_dual_v: head_dim %lld not built (64 and 128 are)", (long long)D);
  MOTIF_REQUIRE(h_q % h_kv == 0, MOTIF_ERR_BAD_CONTRACT, "sdpa_dual_v: H_q=%lld must be a multiple of H_kv=%lld",
                (long long)h_q, (long long)h_kv);
  MOTIF_REQUIRE(h_q / h_kv <= 8, MOTIF_ERR_BAD_CONTRACT, "sdpa_dual_v: GQA factor %lld > 8 not built",
                (long long)(h_q / h_kv));
  MOTIF_REQUIRE(kv_len_dev || (kv_len >= 0 && kv_len <= cap), MOTIF_ERR_BAD_SHAPE,
                "sdpa_dual_v: kv_len=%lld must be in [0, %lld]", (long long)kv_len, (long long)cap);
  MOTIF_REQUIRE(cap < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "sdpa_dual_v: capacity too large");
  return MOTIF_OK;
}

bool al(const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

}  // namespace
}  // namespace motif

using namespace motif;

extern "C" {

size_t motif_sdpa_dual_v_workspace_bytes(int64_t batch, int64_t h_q, int64_t head_dim,
                                         int64_t max_splits) {
  return partial_bytes(batch * h_q, head_dim, max_splits < 1 ? 1 : max_splits);
}

int motif_sdpa_dual_v(int dtype, const void* q, const void* k, const void* v1, const void* v2,
                      float scale, int64_t batch, int64_t h_q, int64_t h_kv, int64_t kv_cap,
                      int64_t head_dim, int64_t kv_len, const int32_t* kv_len_dev, void* y,
                      void* workspace, size_t workspace_bytes, void* stream) {
  MOTIF_REQUIRE(q && k && v1 && v2 && y, MOTIF_ERR_NULL, "sdpa_dual_v: null pointer");
  int rc = check_common(batch, h_q, h_kv, kv_cap, head_dim, kv_len, kv_len_dev);
  if (rc) return rc;
  const int esz = dtype == MOTIF_F32 ? 4 : 2;
  for (const void* p : {q, k, v1, v2})
    MOTIF_REQUIRE(al(p, esz * (int)(head_dim / 32)), MOTIF_ERR_BAD_SHAPE, "sdpa_dual_v: misaligned input");
  AttnArgs a{};
  a.q = q;
  a.q_bstride = h_q * head_dim;
  a.na = (int)(h_q / h_kv);
  a.nb_base = 0;
  a.h_out = (int)h_q;
  a.kA = k;
  a.v1 = v1;
  a.v2 = v2;
  a.h_kv = (int)h_kv;
  a.cap = kv_cap;
  a.gs = 64;
  a.kv_len = (int)kv_len;
  a.kv_len_dev = kv_len_dev;
  a.scale_log2 = scale * kLog2e;
  a.y = y;
  cudaStream_t st = as_stream(stream);
  MOTIF_DISPATCH_FLOAT(dtype, T, return run_generic<T>(16, a, batch, h_q, h_kv, kv_cap, head_dim, kv_len, workspace, workspace_bytes, st));
  return MOTIF_OK;
}

int motif_sdpa_dual_v_q(int dtype, int bits, int group_size, const void* q,
                        const uint32_t* k_data, const void* k_scales, const void* k_biases,
                        const uint32_t* v1_data, const void* v1_scales, const void* v1_biases,
                        const uint32_t* v2_data, const void* v2_scales, const void* v2_biases,
                        float scale, int64_t batch, int64_t h_q, int64_t h_kv, int64_t kv_cap,
                        int64_t head_dim, int64_t kv_len, const int32_t* kv_len_dev, void* y,
                        void* workspace, size_t workspace_bytes, void* stream) {
  MOTIF_REQUIRE(q && k_data && k_scales && k_biases && v1_data && v1_scales && v1_biases &&
                    v2_data && v2_scales && v2_biases && y,
                MOTIF_ERR_NULL, "sdpa_dual_v_q: null pointer");
  MOTIF_REQUIRE(bits == 4 || bits == 8, MOTIF_ERR_BAD_CONTRACT, "sdpa_dual_v_q: bits=%d not in (4, 8)", bits);
  const int64_t D = head_dim;
  MOTIF_REQUIRE(D % 32 == 0 && group_size > 0 && D % group_size == 0, MOTIF_ERR_BAD_CONTRACT,
                "sdpa_dual_v_q: need D %% 32 == 0 and D %% group_size == 0 (D=%lld, group_size=%d)",
                (long long)D, group_size);
  const int64_t cpl = D / 32;
  MOTIF_REQUIRE((32 / bits) % cpl == 0, MOTIF_ERR_BAD_CONTRACT,
                "sdpa_dual_v_q: each lane's qk_per_thread = D/32 channels must come from one packed "
                "uint32, i.e. qk_per_thread | EL_PER_INT (which implies D/32 <= 32/bits); got D=%lld, "
                "bits=%d -> qk_per_thread=%lld, EL_PER_INT=%d",
                (long long)D, bits, (long long)cpl, 32 / bits);
  MOTIF_REQUIRE(group_size % cpl == 0, MOTIF_ERR_BAD_CONTRACT,
                "sdpa_dual_v_q: qk_per_thread | group_size required so a lane's D/32 channels share one "
                "scale/bias group; got D=%lld, group_size=%d -> qk_per_thread=%lld",
                (long long)D, group_size, (long long)cpl);
  int rc = check_common(batch, h_q, h_kv, kv_cap, D, kv_len, kv_len_dev);
  if (rc) return rc;
  AttnArgs a{};
  a.q = q;
  a.q_bstride = h_q * D;
  a.na = (int)(h_q / h_kv);
  a.nb_base = 0;
  a.h_out = (int)h_q;
  a.kA = k_data;
  a.v1 = v1_data;
  a.v2 = v2_data;
  a.kA_s = k_scales;
  a.kA_b = k_biases;
  a.v1_s = v1_scales;
  a.v1_b = v1_biases;
  a.v2_s = v2_scales;
  a.v2_b = v2_biases;
  a.h_kv = (int)h_kv;
  a.cap = kv_cap;
  a.gs = group_size;
  a.kv_len = (int)kv_len;
  a.kv_len_dev = kv_len_dev;
  a.scale_log2 = scale * kLog2e;
  a.y = y;
  cudaStream_t st = as_stream(stream);
  MOTIF_DISPATCH_FLOAT(dtype, T, return run_generic<T>(bits, a, batch, h_q, h_kv, kv_cap, D, kv_len, workspace, workspace_bytes, st));
  return MOTIF_OK;
}

size_t motif_gda_decode_attention_workspace_bytes(int64_t q_heads, int64_t head_dim,
                                                  int64_t max_splits) {
  return partial_bytes(q_heads, head_dim, max_splits < 1 ? 1 : max_splits);
}

int motif_gda_decode_attention(const void* q, const motif_kv4_slots* cache, float scale,
                               int64_t q_groups, int64_t gr, int64_t kv_len,
                               const int32_t* kv_len_dev, const void* subln_w,
                               const float* lambda_full, int64_t lambda_len, float lambda_init,
                               float eps, void* out, void* workspace, size_t workspace_bytes,
                               void* stream) {
  MOTIF_REQUIRE(q && cache && subln_w && lambda_full && out && workspace, MOTIF_ERR_NULL,
                "gda_decode_attention: null pointer");
  const motif_kv4_slots& c = *cache;
  for (int i = 0; i < 4; ++i) MOTIF_REQUIRE(c.data[i], MOTIF_ERR_NULL, "gda_decode_attention: slot %d null", i);
  MOTIF_REQUIRE(c.batch == 1 && c.head_dim == 128, MOTIF_ERR_BAD_CONTRACT,
                "gda_decode_attention: batch 1, head_dim 128 only");
  MOTIF_REQUIRE(c.heads == q_groups, MOTIF_ERR_BAD_CONTRACT,
                "gda_decode_attention: kv heads per slot (%lld) must equal q_groups (%lld)",
                (long long)c.heads, (long long)q_groups);
  MOTIF_REQUIRE(gr == 3 || gr == 4, MOTIF_ERR_BAD_CONTRACT, "gda_decode_attention: gr=%lld not built (3, 4)", (long long)gr);
  MOTIF_REQUIRE(kv_len_dev || (kv_len >= 0 && kv_len <= c.capacity), MOTIF_ERR_BAD_SHAPE,
                "gda_decode_attention: kv_len out of range");
  const int64_t q_origin = q_groups * gr;
  const int64_t q_heads = q_origin + q_groups;
  int lam_mode;
  if (lambda_len == 1) lam_mode = 0;
  else if (lambda_len == q_groups) lam_mode = 1;
  else if (lambda_len == q_origin) lam_mode = 2;
  else return fail(MOTIF_ERR_BAD_SHAPE, "gda_decode_attention: lambda_len %lld", (long long)lambda_len);
  const int bits = c.bits;
  MOTIF_REQUIRE(bits == 16 || ((bits == 4 || bits == 8) && c.scales[0] && c.biases[0] &&
                               (c.group_size == 32 || c.group_size == 64 || c.group_size == 128)),
                MOTIF_ERR_BAD_CONTRACT, "gda_decode_attention: cache bits/group_size");
  const int64_t len_bound = kv_len_dev ? c.capacity : kv_len;
  const int64_t max_splits_ws = workspace_bytes / partial_bytes(q_heads, 128, 1);
  MOTIF_REQUIRE(max_splits_ws >= 1, MOTIF_ERR_WORKSPACE, "gda_decode_attention: workspace too small");
  const int nsplit = choose_splits(q_groups, len_bound, max_splits_ws);

  AttnArgs a{};
  a.q = q;
  a.q_bstride = 0;
  a.na = (int)gr;
  a.nb_base = (int)q_origin;
  a.h_out = (int)q_heads;
  a.kA = c.data[0];
  a.kB = c.data[1];
  a.v1 = c.data[2];
  a.v2 = c.data[3];
  a.kA_s = c.scales[0];
  a.kA_b = c.biases[0];
  a.kB_s = c.scales[1];
  a.kB_b = c.biases[1];
  a.v1_s = c.scales[2];
  a.v1_b = c.biases[2];
  a.v2_s = c.scales[3];
  a.v2_b = c.biases[3];
  a.h_kv = (int)c.heads;
  a.cap = c.capacity;
  a.gs = c.group_size;
  a.kv_len = (int)kv_len;
  a.kv_len_dev = kv_len_dev;
  a.scale_log2 = scale * kLog2e;
  a.force_partials = 1;
  a.ws = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  int rc;
#define MOTIF_FUSED(GR)                                                                    \
  if (bits == 16) rc = launch_split<__half, 128, 16, GR, 1>(a, nsplit, 1, st);            \
  else if (bits == 4) rc = launch_split<__half, 128, 4, GR, 1>(a, nsplit, 1, st);         \
  else rc = launch_split<__half, 128, 8, GR, 1>(a, nsplit, 1, st);                        \
  if (rc) return rc;                                                                      \
  gda_combine_kernel<128, GR><<<q_groups, 256, 0, st>>>(                                  \
      a.ws, nsplit, (int)kv_len, kv_len_dev, (int)q_origin,                               \
      static_cast<const __half*>(subln_w), lambda_full, lam_mode, 1.0f - lambda_init, eps, \
      static_cast<__half*>(out));
  if (gr == 3) {
    MOTIF_FUSED(3)
  } else {
    MOTIF_FUSED(4)
  }
#undef MOTIF_FUSED
  return check_launch("gda decode attention");
}

}  // extern "C"

namespace motif {
namespace {

constexpr int kMaxClusterSplitsForSmem = 8;

// Dynamic shared memory of gda_fused_kernel: the per-warp softmax states, and on the cluster
// path rank 0's slots for every split's partial.
size_t fused_smem_bytes(int heads, bool cluster) {
  return sizeof(float) * ((size_t)kAttnWarps * heads * (2 + 2 * 128) +
                          (cluster ? (size_t)kMaxClusterSplitsForSmem * heads * (2 + 2 * 128) : 0));
}

template <int NA, int NB, bool PAIRED, int PPW, int BITS, int LPG, bool CLUSTER>
cudaError_t launch_fused_one(const FusedArgs& f, dim3 grid, cudaStream_t st) {
  auto kern = gda_fused_kernel<BITS, NA, NB, PAIRED, PPW, LPG, CLUSTER>;
  const size_t smem = fused_smem_bytes(NA + NB, CLUSTER);
  static bool configured = false;  // one attribute call per instantiation
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = grid.x;  // the group's splits form one cluster
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = CLUSTER ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, f);
}

// Largest cluster (splits of one group) the cluster merge takes: 8 CTAs, the portable size;
// MOTIF_ATTN_CLUSTER=0 turns the cluster merge off.
constexpr int kMaxClusterSplits = kMaxClusterSplitsForSmem;

bool cluster_merge_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("MOTIF_ATTN_CLUSTER");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Whether a cluster of `nsplit` CTAs of this instantiation can be resident (cudaOccupancyMaxActiveClusters).
template <int NA, int NB, bool PAIRED, int PPW, int BITS, int LPG>
bool cluster_fits(int nsplit) {
  auto kern = gda_fused_kernel<BITS, NA, NB, PAIRED, PPW, LPG, true>;
  const size_t smem = fused_smem_bytes(NA + NB, true);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, 1);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nsplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return clusters >= 1;
}

// The one-launch attention step for one head layout, dispatched over the cache's bits and group size.
// The launch of one (bits, group size) instantiation: the cluster merge when the splits fit one
// cluster (GDA layout only), else the global merge.
template <int NA, int NB, bool PAIRED, int PPW, int BITS, int LPG>
cudaError_t launch_fused_bits(const FusedArgs& f, dim3 grid, cudaStream_t st) {
  if constexpr (!PAIRED && NB == 1) {
    // Caches of up to 2·kMaxClusterSplits·kMinChunk rows (at most two rounds of rows per
    // split): the splits shrink to one portable cluster of at most 8 CTAs. Larger clusters were
    // slower to schedule than the global merge they replace.
    if (grid.x >= 2 && grid.x <= 2u * kMaxClusterSplits && cluster_merge_enabled()) {
      const dim3 cgrid(grid.x < (unsigned)kMaxClusterSplits ? grid.x : kMaxClusterSplits, grid.y);
      static int fits[kMaxClusterSplits + 1] = {};  // 0 unknown, 1 yes, 2 no (per split count)
      int& fit = fits[cgrid.x];
      if (!fit) fit = cluster_fits<NA, NB, PAIRED, PPW, BITS, LPG>((int)cgrid.x) ? 1 : 2;
      if (fit == 1) return launch_fused_one<NA, NB, PAIRED, PPW, BITS, LPG, true>(f, cgrid, st);
    }
  }
  return launch_fused_one<NA, NB, PAIRED, PPW, BITS, LPG, false>(f, grid, st);
}

template <int NA, int NB, bool PAIRED, int PPW>
cudaError_t launch_fused(const FusedArgs& f, dim3 grid, int bits, int gs, cudaStream_t st) {
  if (bits == 16) return launch_fused_bits<NA, NB, PAIRED, PPW, 16, 8>(f, grid, st);
  if (gs == 32) return bits == 4 ? launch_fused_bits<NA, NB, PAIRED, PPW, 4, 4>(f, grid, st)
                                 : launch_fused_bits<NA, NB, PAIRED, PPW, 8, 4>(f, grid, st);
  if (gs == 64) return bits == 4 ? launch_fused_bits<NA, NB, PAIRED, PPW, 4, 8>(f, grid, st)
                                 : launch_fused_bits<NA, NB, PAIRED, PPW, 8, 8>(f, grid, st);
  return bits == 4 ? launch_fused_bits<NA, NB, PAIRED, PPW, 4, 16>(f, grid, st)
                   : launch_fused_bits<NA, NB, PAIRED, PPW, 8, 16>(f, grid, st);
}

template <int NA, int NB, bool PAIRED, int BITS>
cudaError_t launch_long_bits(const FusedArgs& f, const LongMaps& m, dim3 grid, cudaStream_t st) {
  auto kern = gda_long_kernel<NA, NB, PAIRED, BITS>;
  constexpr int smem = long_smem<BITS>();
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(LongCfg<BITS>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, f, m);
}

template <int NA, int NB, bool PAIRED>
cudaError_t launch_long_one(const FusedArgs& f, const LongMaps& m, dim3 grid, cudaStream_t st) {
  return f.cache.bits == 16 ? launch_long_bits<NA, NB, PAIRED, 16>(f, m, grid, st)
                            : launch_long_bits<NA, NB, PAIRED, 4>(f, m, grid, st);
}

// Caches at least this long (capacity, fp16) take the tensor-core step; MOTIF_LONG_ATTN_MIN_CAP
// overrides it (0 = always, a huge value = never).
int64_t long_min_cap() {
  const char* v = getenv("MOTIF_LONG_ATTN_MIN_CAP");
  return v ? atoll(v) : 2048;
}

// Whether the tensor-core step takes this cache: fp16 rows, or q4 group 64 with the capacity a
// multiple of 4 (scales and biases travel as 16-byte lines of four rows, so a head's rows must
// start on a line), a capacity of at least long_min_cap() rows and 16-byte aligned slots. Host
// arithmetic only; the caches of mlx_motif allocate whole 256-row steps, so the capacity rule
// always holds for them.
bool long_eligible(const motif_kv4_slots& c) {
  if (c.capacity < long_min_cap() || c.heads >= kLErrSlot || c.heads * c.capacity >= (1ll << 31)) return false;
  const bool q4 = c.bits == 4 && c.group_size == 64 && c.capacity % 4 == 0;
  if (c.bits != 16 && !q4) return false;
  for (int i = 0; i < 4; ++i) {
    uintptr_t addr = reinterpret_cast<uintptr_t>(c.data[i]);
    if (c.bits != 16) addr |= reinterpret_cast<uintptr_t>(c.scales[i]) | reinterpret_cast<uintptr_t>(c.biases[i]);
    if (!c.data[i] || addr % 16) return false;
  }
  return true;
}

// The tensor-core step's maps over the four slots, or false when the cache does not fit it.
bool long_maps(const motif_kv4_slots& c, LongMaps& m) {
  if (!long_eligible(c)) return false;
  const uint64_t rows = (uint64_t)(c.heads * c.capacity);
  for (int i = 0; i < 4; ++i) {
    if (c.bits == 16) {
      if (!encode_tma_rows(&m.slot[i], c.data[i], 256, rows, 128, kLT, true)) return false;
    } else {
      if (!encode_tma_rows(&m.slot[i], c.data[i], 64, rows, 64, kLT, false) ||
          !encode_tma_rows(&m.sc[i], c.scales[i], 16, rows / 4, 16, kLT / 4, false) ||
          !encode_tma_rows(&m.bi[i], c.biases[i], 16, rows / 4, 16, kLT / 4, false))
        return false;
    }
  }
  return true;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        n <= 0)
      n = 148;
  }
  return n;
}

// One CTA per SM (the ring takes ~210 KB of shared memory), all in one wave.
int long_splits(int64_t groups, int64_t max_splits_ws) {
  int64_t n = sm_count() / (groups < 1 ? 1 : groups);
  if (n > max_splits_ws) n = max_splits_ws;
  if (n > kMaxSplits) n = kMaxSplits;
  return (int)(n < 1 ? 1 : n);
}

int check_fused_cache(const motif_kv4_slots& c, int64_t groups, const char* who) {
  for (int i = 0; i < 4; ++i) MOTIF_REQUIRE(c.data[i], MOTIF_ERR_NULL, "%s: slot %d null", who, i);
  MOTIF_REQUIRE(c.batch == 1 && c.head_dim == 128, MOTIF_ERR_BAD_CONTRACT, "%s: batch 1, head_dim 128 only", who);
  MOTIF_REQUIRE(c.heads == groups && groups > 0, MOTIF_ERR_BAD_CONTRACT,
                "%s: kv heads per slot (%lld) must equal the groups (%lld)", who, (long long)c.heads,
                (long long)groups);
  MOTIF_REQUIRE(c.capacity > 0 && c.capacity < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "%s: capacity", who);
  const int bits = c.bits;
  MOTIF_REQUIRE(bits == 16 || ((bits == 4 || bits == 8) && c.scales[0] && c.biases[0] && c.scales[1] && c.biases[1] &&
                               c.scales[2] && c.biases[2] && c.scales[3] && c.biases[3] &&
                               (c.group_size == 32 || c.group_size == 64 || c.group_size == 128)),
                MOTIF_ERR_BAD_CONTRACT, "%s: cache bits/group_size", who);
  MOTIF_REQUIRE(groups * sizeof(int) <= kFusedCtlBytes, MOTIF_ERR_BAD_SHAPE, "%s: too many groups", who);
  return MOTIF_OK;
}

}  // namespace
}  // namespace motif

extern "C" {

int motif_decode_step_kernel(const motif_kv4_slots* cache) {
  if (!cache) return -fail(MOTIF_ERR_NULL, "decode_step_kernel: null cache");
  const motif_kv4_slots& c = *cache;
  if (int rc = check_fused_cache(c, c.heads, "decode_step_kernel")) return -rc;
  return long_eligible(c) ? MOTIF_ATTN_KERNEL_TCGEN05 : MOTIF_ATTN_KERNEL_SPLIT;
}

size_t motif_gda_decode_step_workspace_bytes(int64_t q_heads, int64_t head_dim, int64_t max_splits) {
  if (q_heads <= 0 || head_dim <= 0 || max_splits <= 0) return 0;
  return kFusedCtlBytes + partial_bytes(q_heads, head_dim, max_splits < kMaxSplits ? max_splits : kMaxSplits);
}

int motif_gda_decode_step(const void* qkv, const float* inv_freq, const motif_kv4_slots* cache,
                          const int32_t* pos_len, float scale, int64_t q_groups, int64_t gr,
                          const void* subln_w, const float* lambda_full, int64_t lambda_len,
                          float lambda_init, float eps, void* out, void* workspace,
                          size_t workspace_bytes, void* stream) {
  MOTIF_REQUIRE(qkv && inv_freq && cache && pos_len && subln_w && lambda_full && out && workspace, MOTIF_ERR_NULL,
                "gda_decode_step: null pointer");
  const motif_kv4_slots& c = *cache;
  for (int i = 0; i < 4; ++i) MOTIF_REQUIRE(c.data[i], MOTIF_ERR_NULL, "gda_decode_step: slot %d null", i);
  MOTIF_REQUIRE(c.batch == 1 && c.head_dim == 128, MOTIF_ERR_BAD_CONTRACT, "gda_decode_step: batch 1, head_dim 128 only");
  MOTIF_REQUIRE(c.heads == q_groups && q_groups > 0, MOTIF_ERR_BAD_CONTRACT,
                "gda_decode_step: kv heads per slot (%lld) must equal q_groups (%lld)", (long long)c.heads,
                (long long)q_groups);
  MOTIF_REQUIRE(gr == 3 || gr == 4, MOTIF_ERR_BAD_CONTRACT, "gda_decode_step: gr=%lld not built (3, 4)", (long long)gr);
  MOTIF_REQUIRE(c.capacity > 0 && c.capacity < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "gda_decode_step: capacity");
  const int64_t q_origin = q_groups * gr;
  const int64_t q_heads = q_origin + q_groups;
  int lam_mode;
  if (lambda_len == 1) lam_mode = 0;
  else if (lambda_len == q_groups) lam_mode = 1;
  else if (lambda_len == q_origin) lam_mode = 2;
  else return fail(MOTIF_ERR_BAD_SHAPE, "gda_decode_step: lambda_len %lld", (long long)lambda_len);
  const int bits = c.bits;
  MOTIF_REQUIRE(bits == 16 || ((bits == 4 || bits == 8) && c.scales[0] && c.biases[0] && c.scales[1] && c.biases[1] &&
                               c.scales[2] && c.biases[2] && c.scales[3] && c.biases[3] &&
                               (c.group_size == 32 || c.group_size == 64 || c.group_size == 128)),
                MOTIF_ERR_BAD_CONTRACT, "gda_decode_step: cache bits/group_size");
  MOTIF_REQUIRE(q_groups * sizeof(int) <= kFusedCtlBytes, MOTIF_ERR_BAD_SHAPE, "gda_decode_step: too many groups");
  MOTIF_REQUIRE(workspace_bytes > kFusedCtlBytes, MOTIF_ERR_WORKSPACE, "gda_decode_step: workspace too small");
  const int64_t max_splits_ws = (workspace_bytes - kFusedCtlBytes) / partial_bytes(q_heads, 128, 1);
  MOTIF_REQUIRE(max_splits_ws >= 1, MOTIF_ERR_WORKSPACE, "gda_decode_step: workspace too small");
  const int nsplit = choose_splits(q_groups, c.capacity, max_splits_ws);

  FusedArgs f{};
  f.qkv = static_cast<const __half*>(qkv);
  f.inv_freq = inv_freq;
  f.q_heads = (int)q_heads;
  f.q_origin = (int)q_origin;
  f.groups = (int)q_groups;
  f.cache = c;
  f.pos_len = pos_len;
  f.scale_log2 = scale * kLog2e;
  f.subln_w = static_cast<const __half*>(subln_w);
  f.lam = lambda_full;
  f.lam_mode = lam_mode;
  f.out_scale = 1.0f - lambda_init;
  f.eps = eps;
  f.out = static_cast<__half*>(out);
  f.counters = static_cast<int*>(workspace);
  f.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + kFusedCtlBytes);
  cudaStream_t st = as_stream(stream);
  cudaError_t e;
  LongMaps lm;
  if (long_maps(c, lm)) {
    const dim3 grid(long_splits(q_groups, max_splits_ws), (unsigned)q_groups);
    e = gr == 3 ? launch_long_one<3, 1, false>(f, lm, grid, st) : launch_long_one<4, 1, false>(f, lm, grid, st);
  } else {
    const dim3 grid(nsplit, (unsigned)q_groups);
    e = gr == 3 ? launch_fused<3, 1, false, 4>(f, grid, c.bits, c.group_size, st)
                : launch_fused<4, 1, false, 4>(f, grid, c.bits, c.group_size, st);
  }
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "gda_decode_step: launch: %s", cudaGetErrorString(e));
  return check_launch("gda decode step");
}

int motif_vanilla_decode_step(const void* qkv, const float* inv_freq, const motif_kv4_slots* cache,
                              const int32_t* pos_len, float scale, int64_t kv_heads, int64_t n_rep,
                              const void* subln_w, const float* lambda_full, float lambda_init, float eps,
                              void* out, void* workspace, size_t workspace_bytes, void* stream) {
  MOTIF_REQUIRE(qkv && inv_freq && cache && pos_len && subln_w && lambda_full && out && workspace, MOTIF_ERR_NULL,
                "vanilla_decode_step: null pointer");
  MOTIF_REQUIRE(n_rep == 1 || n_rep == 2 || n_rep == 4, MOTIF_ERR_BAD_CONTRACT,
                "vanilla_decode_step: n_rep=%lld not built (1, 2, 4)", (long long)n_rep);
  const motif_kv4_slots& c = *cache;
  if (int rc = check_fused_cache(c, kv_heads, "vanilla_decode_step")) return rc;
  const int64_t q_heads = 2 * kv_heads * n_rep;  // interleaved q1/q2 stripes
  MOTIF_REQUIRE(workspace_bytes > kFusedCtlBytes, MOTIF_ERR_WORKSPACE, "vanilla_decode_step: workspace too small");
  const int64_t max_splits_ws = (workspace_bytes - kFusedCtlBytes) / partial_bytes(q_heads, 128, 1);
  MOTIF_REQUIRE(max_splits_ws >= 1, MOTIF_ERR_WORKSPACE, "vanilla_decode_step: workspace too small");
  const int nsplit = choose_splits(kv_heads, c.capacity, max_splits_ws);
  FusedArgs f{};
  f.qkv = static_cast<const __half*>(qkv);
  f.inv_freq = inv_freq;
  f.q_heads = (int)q_heads;
  f.q_origin = 0;
  f.groups = (int)kv_heads;
  f.cache = c;
  f.pos_len = pos_len;
  f.scale_log2 = scale * kLog2e;
  f.subln_w = static_cast<const __half*>(subln_w);
  f.lam = lambda_full;
  f.lam_mode = 0;
  f.out_scale = 1.0f - lambda_init;
  f.eps = eps;
  f.out = static_cast<__half*>(out);
  f.counters = static_cast<int*>(workspace);
  f.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + kFusedCtlBytes);
  cudaStream_t st = as_stream(stream);
  cudaError_t e;
  LongMaps lm;
  if (long_maps(c, lm)) {
    const dim3 grid(long_splits(kv_heads, max_splits_ws), (unsigned)kv_heads);
    if (n_rep == 1) e = launch_long_one<1, 1, true>(f, lm, grid, st);
    else if (n_rep == 2) e = launch_long_one<2, 2, true>(f, lm, grid, st);
    else e = launch_long_one<4, 4, true>(f, lm, grid, st);
  } else {
    const dim3 grid(nsplit, (unsigned)kv_heads);
    if (n_rep == 1) e = launch_fused<1, 1, true, 4>(f, grid, c.bits, c.group_size, st);
    else if (n_rep == 2) e = launch_fused<2, 2, true, 4>(f, grid, c.bits, c.group_size, st);
    else e = launch_fused<4, 4, true, 2>(f, grid, c.bits, c.group_size, st);
  }
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "vanilla_decode_step: launch: %s", cudaGetErrorString(e));
  return check_launch("vanilla decode step");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of motif_sdpa_dual_v.
//
// Some callers cannot call cudaMalloc at all: a plugin whose device memory
// belongs to the host framework's own allocator, and hot paths that must
// not take cudaMalloc's implicit device synchronisation. For them the split-KV
// partials live in this file-scope device array instead of a caller
// workspace. It is sized once for the library (kStaticScratchBytes) and
// every GPU that loads the library holds it until the process exits.
// ---------------------------------------------------------------------------
namespace motif {
namespace {

constexpr size_t kStaticScratchBytes = 4u << 20;  // 4 MiB of split partials
static __device__ __align__(256) float g_attn_scratch[kStaticScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
// One resolved address per device. Atomic, so host threads making their first call on the
// same device at the same time do not race: each may resolve it, all store the same value.
static std::atomic<void*> g_scratch_ptr[kMaxDevices];

// Host code may not use g_attn_scratch as a device address: it names the
// host-side stand-in. Resolve the device address once per device, with that
// device current.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "sdpa_dual_v_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(MOTIF_ERR_CUDA, "sdpa_dual_v_static: device %d out of range", dev);
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p)
      return fail(MOTIF_ERR_CUDA, "sdpa_dual_v_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return MOTIF_OK;
}

}  // namespace
}  // namespace motif

extern "C" {

size_t motif_sdpa_dual_v_static_scratch_bytes(void) { return motif::kStaticScratchBytes; }

int motif_sdpa_dual_v_static(int dtype, const void* q, const void* k, const void* v1, const void* v2,
                             float scale, int64_t batch, int64_t h_q, int64_t h_kv, int64_t kv_cap,
                             int64_t head_dim, int64_t kv_len, const int32_t* kv_len_dev, void* y,
                             void* stream) {
  MOTIF_REQUIRE(q && k && v1 && v2 && y, MOTIF_ERR_NULL, "sdpa_dual_v_static: null pointer");
  int rc = check_common(batch, h_q, h_kv, kv_cap, head_dim, kv_len, kv_len_dev);
  if (rc) return rc;
  const size_t two_splits = partial_bytes(batch * h_q, head_dim, 2);
  MOTIF_REQUIRE(two_splits <= kStaticScratchBytes, MOTIF_ERR_WORKSPACE,
                "sdpa_dual_v_static: batch*h_q=%lld rows at head_dim %lld need %zu bytes of split "
                "scratch, more than the %zu-byte static array; call motif_sdpa_dual_v with a workspace",
                (long long)(batch * h_q), (long long)head_dim, two_splits, kStaticScratchBytes);
  void* scratch = nullptr;
  rc = static_scratch(&scratch);
  if (rc) return rc;
  return motif_sdpa_dual_v(dtype, q, k, v1, v2, scale, batch, h_q, h_kv, kv_cap, head_dim, kv_len,
                           kv_len_dev, y, scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
