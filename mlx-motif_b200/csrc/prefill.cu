// Prompt (prefill) attention on the 5th-generation tensor cores, and the differential combine
// that follows it.
//
// Reference: a prompt forward runs mx.fast.scaled_dot_product_attention with the causal mask
// over the cache fetched after the append — for the grouped model the origin heads against k1
// and the noise heads against k2, each with both value slots (the shared-QK dual-V pair of
// src/mlx_motif/model.py:769-807), and for the vanilla model the four per-slab SDPAs of
// _forward_vanilla (model.py:486-559: q1 heads on k1, q2 heads on k2, each against both value
// slabs, native GQA). Both reduce to one operation per query head: causal softmax(q·kᵀ·scale)
// over one key slot, applied to the 256-wide [v1 | v2] row; then gda_post_split
// (kernels/gda.py:223-282) or the vanilla (o1 − λ·o2) · SubLN · (1 − λ_init).
//
// prefill_attn_kernel: one CTA per (128-query tile, query head), FlashAttention-style over
// 64-position key tiles:
//   warp 0      TMA: the Q tile (128 rows × 128 dims, two 128-byte-swizzled halves), then per
//               key tile the K tile (64 × 128) and the V tile (64 positions × [v1 | v2]) into
//               two-stage rings.
//   warp 1      allocates tensor memory (S: two 64-column buffers, O: 256 columns) and one
//               lane issues tcgen05.mma: S_j = Q·K_jᵀ (M 128, N 64, K 128, both K-major) one
//               tile ahead, and O += P_j·V_j (M 128, N 256, K 64; P K-major from shared memory,
//               V MN-major straight from the cache rows).
//   warps 2..5  one thread per query row: read S_j from tensor memory, apply the causal mask
//               and the online softmax, write P_j (fp16) to shared memory in the K-major
//               swizzled layout. The running maximum is re-based lazily: O (in tensor memory)
//               is rescaled only when a row's maximum grew by more than 2^8, so P stays
//               ≤ 256 and the result is exact. At the end O / l is written as fp16.
// All waits are bounded; a wait that gives up sets the abort flag and the error word, and the
// CTA drains its loads, gets its commits and frees tensor memory before it exits.
#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace motif {

bool encode_tma_rows(CUtensorMap* m, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_inner,
                     uint32_t box_rows, bool swizzle128);

namespace {

constexpr int kQT = 128;  // query rows per CTA
constexpr int kKT = 64;   // key positions per tile
constexpr int kPAThreads = 192;

struct PrefillArgs {
  CUtensorMap tm_q;     // q head-major: (q_heads·S) rows × 256 B; box 128 B × 128 rows, 128-byte swizzle
  CUtensorMap tm_k[2];  // k1, k2 slots: (heads·cap) rows × 256 B; box 128 B × 64 rows, swizzled
  CUtensorMap tm_v[2];  // v1, v2 slots: same
  __half* out;          // (S, q_heads, 256) token-major
  int S, QH, cap, off;  // queries, query heads, cache capacity, absolute position of query 0
  int mode, gr, q_origin;
  float scale_log2;
  int* err;
  float* part;  // split-KV partials (gridDim.z > 1): [QH][splits][S][kPartStride] fp32
  const int32_t* off_dev;  // when set, the position of query 0 is read here (graph replays)
};

// A split's partial state of one (head, row): unnormalised O (256), its reference maximum
// (log2 domain) and Σp, padded to a 16-byte multiple.
constexpr int kPartStride = 260;
constexpr int kMaxSplits = 16;

// shared-memory map (bytes from a 1024-byte aligned base)
constexpr int kOffQ = 0;            // 2 × 16 KB
constexpr int kOffK = 32768;        // 2 stages × 2 × 8 KB
constexpr int kOffV = 65536;        // 2 stages × 4 × 8 KB
constexpr int kOffP = 131072;       // 2 × 16 KB
constexpr int kOffBar = 163840;     // 15 barriers
constexpr int kNumBars = 15;
constexpr int kPASmem = kOffBar + kNumBars * 8 + 16 + 1024;

// tensor-memory columns
constexpr uint32_t kColS = 0;    // S_j at kColS + 64·(j mod 2)
constexpr uint32_t kColO = 256;  // O: 256 columns

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(kPAThreads, 1) prefill_attn_kernel(const __grid_constant__ PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = tc::smem_addr(smem);
  const uint32_t bar = sb + kOffBar;
  const uint32_t q_full = bar;
  auto k_full = [&](int s) { return bar + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bar + 8u * (3 + s); };
  auto v_full = [&](int s) { return bar + 8u * (5 + s); };
  auto v_empty = [&](int s) { return bar + 8u * (7 + s); };
  auto s_full = [&](int s) { return bar + 8u * (9 + s); };
  auto p_full = [&](int s) { return bar + 8u * (11 + s); };
  const uint32_t o_bar = bar + 8u * 13;
  const uint32_t drain = bar + 8u * 14;  // the MMA thread's last commit: nothing in flight after it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest (last) query tiles first: the causal work grows with the tile index
  const int tile = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y;
  const int q0 = tile * kQT;
  const int rows = min(kQT, a.S - q0);
  int kslot, g;
  if (a.mode == 0) {
    kslot = h < a.q_origin ? 0 : 1;
    g = h < a.q_origin ? h / a.gr : h - a.q_origin;
  } else {
    kslot = h & 1;
    g = (h >> 1) / a.gr;
  }
  const int off = a.off_dev ? *a.off_dev : a.off;
  if (off < 0 || off + a.S > a.cap) {  // a device offset outside the cache: nothing is read
    if (threadIdx.x == 0 && a.err) atomicExch(a.err, 1);
    return;
  }
  const int kv_end = off + q0 + rows;  // keys [0, kv_end) are visible to some row of the tile
  const int nt_all = (kv_end + kKT - 1) / kKT;
  // Split-KV (short blocks): this CTA takes key tiles [j0, j0 + nt). Below, j counts this
  // CTA's tiles (ring stages, barrier parities).
  const int nsplit = gridDim.z, split = blockIdx.z;
  const int j0 = (int)((int64_t)split * nt_all / nsplit);
  const int nt = (int)((int64_t)(split + 1) * nt_all / nsplit) - j0;
  if (nt <= 0) {  // more splits than key tiles (a device offset below the launch's bound): empty state
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
      float* pdst = a.part + (((int64_t)h * nsplit + split) * a.S + q0 + r) * kPartStride;
      pdst[256] = -INFINITY;
      pdst[257] = 0.f;
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) tc::mbar_init(bar + 8u * i, (i == 11 || i == 12) ? 4 : 1);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_addr(tmem_slot), 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer ----
      const int krow = g * a.cap;
      tc::mbar_expect_tx(q_full, 2 * 16384);
      tc::tma_load_2d(sb + kOffQ, &a.tm_q, 0, h * a.S + q0, q_full);
      tc::tma_load_2d(sb + kOffQ + 16384, &a.tm_q, 128, h * a.S + q0, q_full);
      int k_iss = 0, v_iss = 0;
      for (int j = 0; j < nt; ++j) {
        const int s = j & 1;
        const uint32_t r = j >> 1;
        if (j >= 2 && !tc::mbar_wait(k_empty(s), (r - 1) & 1)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        const uint32_t kb = sb + kOffK + s * 16384;
        tc::mbar_expect_tx(k_full(s), 16384);
        const int kpos = krow + (j0 + j) * kKT;
        tc::tma_load_2d(kb, &a.tm_k[kslot], 0, kpos, k_full(s));
        tc::tma_load_2d(kb + 8192, &a.tm_k[kslot], 128, kpos, k_full(s));
        k_iss = j + 1;
        if (j >= 2 && !tc::mbar_wait(v_empty(s), (r - 1) & 1)) { *abort_flag = 1; break; }
        const uint32_t vb = sb + kOffV + s * 32768;
        tc::mbar_expect_tx(v_full(s), 32768);
        tc::tma_load_2d(vb, &a.tm_v[0], 0, kpos, v_full(s));
        tc::tma_load_2d(vb + 8192, &a.tm_v[0], 128, kpos, v_full(s));
        tc::tma_load_2d(vb + 16384, &a.tm_v[1], 0, kpos, v_full(s));
        tc::tma_load_2d(vb + 24576, &a.tm_v[1], 128, kpos, v_full(s));
        v_iss = j + 1;
      }
      // drain: the loads issued last on each stage have landed before the CTA may exit
      if (!tc::mbar_wait(q_full, 0)) *abort_flag = 1;
      for (int j = k_iss > 2 ? k_iss - 2 : 0; j < k_iss; ++j)
        if (!tc::mbar_wait(k_full(j & 1), (j >> 1) & 1)) *abort_flag = 1;
      for (int j = v_iss > 2 ? v_iss - 2 : 0; j < v_iss; ++j)
        if (!tc::mbar_wait(v_full(j & 1), (j >> 1) & 1)) *abort_flag = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer ----
      constexpr uint32_t idesc_qk = tc::idesc_f16_f32(kQT, kKT);
      constexpr uint32_t idesc_pv = tc::idesc_f16_f32(kQT, 256, true);
      bool ok = tc::mbar_wait(q_full, 0);
      auto issue_qk = [&](int j) -> bool {
        const int s = j & 1;
        if (!tc::mbar_wait(k_full(s), (j >> 1) & 1)) return false;
        tc::tc_fence_after();
        const uint32_t kb = sb + kOffK + s * 16384;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc::mma_f16(tmem + kColS + 64 * s,
                      tc::desc_kmajor_sw128(sb + kOffQ + (kk >> 2) * 16384 + (kk & 3) * 32),
                      tc::desc_kmajor_sw128(kb + (kk >> 2) * 8192 + (kk & 3) * 32), idesc_qk, kk > 0);
        tc::mma_commit(s_full(s));
        tc::mma_commit(k_empty(s));
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; ok && j < nt; ++j) {
        if (*abort_flag) break;
        if (j + 1 < nt && !issue_qk(j + 1)) { ok = false; break; }
        const int s = j & 1;
        if (!tc::mbar_wait(p_full(s), (j >> 1) & 1) || !tc::mbar_wait(v_full(s), (j >> 1) & 1)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t pb = sb + kOffP + s * 16384, vb = sb + kOffV + s * 32768;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_f16(tmem + kColO, tc::desc_kmajor_sw128(pb + kk * 32),
                      tc::desc_mnmajor_sw128(vb + kk * 2048, 8192, 1024), idesc_pv, (j | kk) != 0);
        tc::mma_commit(o_bar);
        tc::mma_commit(v_empty(s));
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued completes before tensor memory can be freed (on abort
      // the softmax warps time out on the tiles that never come, each wait bounded)
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0)) *abort_flag = 1;
    }
    __syncwarp();
  } else {  // ---- softmax + epilogue: one thread per query row ----
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int qa = off + q0 + r;  // absolute position of this row's query
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    float m_ref = -INFINITY, l = 0.f;
    bool alive = true;
    for (int j = 0; j < nt && alive; ++j) {
      const int s = j & 1;
      const bool got = tc::mbar_wait(s_full(s), (j >> 1) & 1);
      if (__any_sync(0xffffffffu, !got || *abort_flag)) {
        *abort_flag = 1;
        alive = false;
        break;
      }
      tc::tc_fence_after();
      uint32_t sv[2][32];
      tc::tmem_ld32(trow + kColS + 64 * s, sv[0]);
      tc::tmem_ld32(trow + kColS + 64 * s + 32, sv[1]);
      tc::tmem_ld_wait();
      const int p0 = (j0 + j) * kKT;
      float x[64];
      float m_tile = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        x[c] = (p0 + c <= qa) ? __uint_as_float(sv[c >> 5][c & 31]) * a.scale_log2 : -INFINITY;
        m_tile = fmaxf(m_tile, x[c]);
      }
      const bool need = m_tile > m_ref + 8.f;
      float factor = 1.f;
      if (need) {
        factor = exp2f(m_ref - m_tile);  // 0 on the first tile (m_ref = -inf)
        m_ref = m_tile;
      }
      l *= factor;
      // a row with no visible key yet (a later split's first tiles) keeps m_ref = -inf and p = 0
      const float mb = m_ref == -INFINITY ? 0.f : m_ref;
      uint32_t pk[32];
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const __half2 hp = __floats2half2_rn(exp2f(x[c] - mb), exp2f(x[c + 1] - mb));
        const float2 fp = __half22float2(hp);
        psum += fp.x + fp.y;
        pk[c >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
      }
      l += psum;
      // O and the P buffer are free once PV(j-1) has completed
      if (j > 0) {
        const bool done = tc::mbar_wait(o_bar, (j - 1) & 1);
        if (__any_sync(0xffffffffu, !done)) {
          *abort_flag = 1;
          alive = false;
          break;
        }
        tc::tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int cb = 0; cb < 8; ++cb) {
            uint32_t ov[32];
            tc::tmem_ld32(trow + kColO + cb * 32, ov);
            tc::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * factor);
            tc::tmem_st32(trow + kColO + cb * 32, ov);
          }
          tc::tmem_st_wait();
        }
      }
      uint8_t* prow = smem + kOffP + s * 16384 + r * 128;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        *reinterpret_cast<uint4*>(prow + ((c8 ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c8], pk[4 * c8 + 1], pk[4 * c8 + 2], pk[4 * c8 + 3]);
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(p_full(s));
    }
    // epilogue: O / l once the last PV has completed
    const bool fin = alive && __all_sync(0xffffffffu, tc::mbar_wait(o_bar, (nt - 1) & 1));
    if (!fin) *abort_flag = 1;
    tc::tc_fence_after();
    const bool live = fin && r < rows;
    const float inv_l = l > 0.f ? 1.f / l : 0.f;
    __half* dst = a.out + ((int64_t)(q0 + r) * a.QH + h) * 256;
    float* pdst = nsplit > 1 ? a.part + (((int64_t)h * nsplit + split) * a.S + q0 + r) * kPartStride : nullptr;
    if (nsplit > 1 && live) {
      pdst[256] = m_ref;
      pdst[257] = l;
    }
#pragma unroll 1
    for (int cb = 0; cb < 8; ++cb) {
      uint32_t ov[32];
      tc::tmem_ld32(trow + kColO + cb * 32, ov);
      tc::tmem_ld_wait();
      if (nsplit > 1) {  // unnormalised O of this split, merged by prefill_merge_kernel
        if (live)
#pragma unroll
          for (int v = 0; v < 8; ++v)
            *reinterpret_cast<float4*>(pdst + cb * 32 + v * 4) =
                make_float4(__uint_as_float(ov[4 * v]), __uint_as_float(ov[4 * v + 1]),
                            __uint_as_float(ov[4 * v + 2]), __uint_as_float(ov[4 * v + 3]));
      } else if (live) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 o;
          o.x = pack_half2(__uint_as_float(ov[8 * v + 0]) * inv_l, __uint_as_float(ov[8 * v + 1]) * inv_l);
          o.y = pack_half2(__uint_as_float(ov[8 * v + 2]) * inv_l, __uint_as_float(ov[8 * v + 3]) * inv_l);
          o.z = pack_half2(__uint_as_float(ov[8 * v + 4]) * inv_l, __uint_as_float(ov[8 * v + 5]) * inv_l);
          o.w = pack_half2(__uint_as_float(ov[8 * v + 6]) * inv_l, __uint_as_float(ov[8 * v + 7]) * inv_l);
          *reinterpret_cast<uint4*>(dst + cb * 32 + v * 8) = o;
        }
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag && a.err) atomicExch(a.err, 1);
}

// Merge of the split-KV partials: per (row, head) the splits' states are rescaled to their
// common maximum, O = Σ w·O_s / Σ w·l_s, rounded to fp16 like the one-CTA path's output.
__global__ void __launch_bounds__(256) prefill_merge_kernel(const float* __restrict__ part, int nsplit, int S, int QH,
                                                            __half* __restrict__ out) {
  const int row = blockIdx.x, h = blockIdx.y, c = threadIdx.x;
  const int64_t sstride = (int64_t)S * kPartStride;
  const float* base = part + ((int64_t)h * nsplit * S + row) * kPartStride;
  float M = -INFINITY;
  for (int i = 0; i < nsplit; ++i) M = fmaxf(M, base[i * sstride + 256]);
  float L = 0.f, o = 0.f;
  for (int i = 0; i < nsplit; ++i) {
    const float* p = base + i * sstride;
    const float m = p[256];
    if (m == -INFINITY) continue;  // a split that saw no key of this row (its O is not written)
    const float w = exp2f(m - M);
    L += w * p[257];
    o += w * p[c];
  }
  out[((int64_t)row * QH + h) * 256 + c] = __float2half_rn(L > 0.f ? o * (1.f / L) : 0.f);
}

// ---- the differential combine over rows -----------------------------------------------------
template <int N>
__device__ __forceinline__ void block_sum_n(float (&v)[N], float* scratch /* [8][N] */) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < N; ++j) scratch[warp * N + j] = v[j];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += scratch[w * N + j];
    v[j] = t;
  }
}

// GDA (PAIRED false): group g = origin heads g·GR + j and noise head q_origin + g,
//   out = fp16((o − λ·n) · rsqrt(mean d² + eps) · w · (1 − λ_init)), as gda_post_split.
// Vanilla (PAIRED true): pairs i = g·GR + j of signal head 2i and noise head 2i + 1, rounded
//   where _forward_vanilla's fp16 arrays round (model.py:553-557).
// One CTA of 256 threads (one per channel) per (row, group); o (S, QH, 256), y (S, q_out, 256).
template <int GR, bool PAIRED>
__global__ void __launch_bounds__(256) prefill_post_kernel(const __half* __restrict__ o, int QH, int q_origin,
                                                           const __half* __restrict__ subln_w,
                                                           const float* __restrict__ lam, int lam_mode,
                                                           float out_scale, float eps, __half* __restrict__ y) {
  __shared__ float scratch[8 * GR];
  const int srow = blockIdx.x, g = blockIdx.y, ch = threadIdx.x;
  const __half* base = o + (int64_t)srow * QH * 256 + ch;
  float d[GR], ssq[GR];
  if constexpr (PAIRED) {
    const float lam16 = __half2float(__float2half_rn(lam[0]));
#pragma unroll
    for (int j = 0; j < GR; ++j) {
      const int i = g * GR + j;
      const float o1 = __half2float(base[(2 * i) * 256]), o2 = __half2float(base[(2 * i + 1) * 256]);
      d[j] = round_through<__half>(o1 - round_through<__half>(lam16 * o2));
      ssq[j] = d[j] * d[j];
    }
  } else {
    const float n = __half2float(base[(q_origin + g) * 256]);
#pragma unroll
    for (int j = 0; j < GR; ++j) {
      const int h = g * GR + j;
      const float l = lam[lam_mode == 0 ? 0 : (lam_mode == 1 ? g : h)];
      d[j] = __half2float(base[h * 256]) - l * n;
      ssq[j] = d[j] * d[j];
    }
  }
  block_sum_n<GR>(ssq, scratch);
  const float w = __half2float(subln_w[ch]);
  const int out_heads = PAIRED ? QH / 2 : q_origin;
  __half* dst = y + (int64_t)srow * out_heads * 256 + ch;
#pragma unroll
  for (int j = 0; j < GR; ++j) {
    const float inv = rsqrtf(ssq[j] / 256.f + eps);
    if constexpr (PAIRED) {
      const float os16 = __half2float(__float2half_rn(out_scale));
      dst[(g * GR + j) * 256] = __float2half_rn(round_through<__half>(d[j] * inv * w) * os16);
    } else {
      dst[(g * GR + j) * 256] = __float2half_rn(d[j] * inv * w * out_scale);
    }
  }
}

template <bool PAIRED>
int launch_post(int gr, dim3 grid, cudaStream_t st, const __half* o, int QH, int q_origin, const __half* w,
                const float* lam, int lam_mode, float out_scale, float eps, __half* y) {
  switch (gr) {
    case 1: prefill_post_kernel<1, PAIRED><<<grid, 256, 0, st>>>(o, QH, q_origin, w, lam, lam_mode, out_scale, eps, y); break;
    case 2: prefill_post_kernel<2, PAIRED><<<grid, 256, 0, st>>>(o, QH, q_origin, w, lam, lam_mode, out_scale, eps, y); break;
    case 3: prefill_post_kernel<3, PAIRED><<<grid, 256, 0, st>>>(o, QH, q_origin, w, lam, lam_mode, out_scale, eps, y); break;
    case 4: prefill_post_kernel<4, PAIRED><<<grid, 256, 0, st>>>(o, QH, q_origin, w, lam, lam_mode, out_scale, eps, y); break;
    default: return fail(MOTIF_ERR_BAD_CONTRACT, "prefill_post: gr=%d not built (1..4)", gr);
  }
  return check_launch("prefill_post");
}

}  // namespace
}  // namespace motif

using namespace motif;

namespace {
int device_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        n <= 0)
      n = 148;
  }
  return n;
}

int prefill_attention(const void* q, int64_t seq, int64_t q_heads, const motif_kv4_slots* cache, int64_t offset,
                      const int32_t* offset_dev, int mode, int64_t gr, float scale, void* out, void* workspace,
                      size_t workspace_bytes, int* err, void* stream) {
  MOTIF_REQUIRE(q && cache && out, MOTIF_ERR_NULL, "prefill_attention: null pointer");
  const motif_kv4_slots& c = *cache;
  for (int i = 0; i < 4; ++i) MOTIF_REQUIRE(c.data[i], MOTIF_ERR_NULL, "prefill_attention: slot %d null", i);
  MOTIF_REQUIRE(c.bits == 16 && c.batch == 1 && c.head_dim == 128, MOTIF_ERR_BAD_CONTRACT,
                "prefill_attention: fp16 4-slot cache, batch 1, head_dim 128 (bits %d)", c.bits);
  MOTIF_REQUIRE(mode == 0 || mode == 1, MOTIF_ERR_BAD_CONTRACT, "prefill_attention: mode %d", mode);
  MOTIF_REQUIRE(seq >= 1 && offset >= 0 && offset + seq <= c.capacity && gr >= 1, MOTIF_ERR_BAD_SHAPE,
                "prefill_attention: rows [%lld, %lld) outside capacity %lld", (long long)offset,
                (long long)(offset + seq), (long long)c.capacity);
  const int64_t G = c.heads;
  const int64_t want = mode == 0 ? G * (gr + 1) : 2 * G * gr;
  MOTIF_REQUIRE(q_heads == want, MOTIF_ERR_BAD_CONTRACT,
                "prefill_attention: %lld query heads, expected %lld for %lld kv heads per slot and gr %lld",
                (long long)q_heads, (long long)want, (long long)G, (long long)gr);
  MOTIF_REQUIRE(q_heads * seq < (1ll << 31) && G * c.capacity < (1ll << 31), MOTIF_ERR_BAD_SHAPE,
                "prefill_attention: too many rows");
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) |
                       reinterpret_cast<uintptr_t>(c.data[0]) | reinterpret_cast<uintptr_t>(c.data[1]) |
                       reinterpret_cast<uintptr_t>(c.data[2]) | reinterpret_cast<uintptr_t>(c.data[3]);
  MOTIF_REQUIRE(al % 16 == 0, MOTIF_ERR_BAD_CONTRACT, "prefill_attention: operands must be 16-byte aligned");
  PrefillArgs a{};
  bool enc = encode_tma_rows(&a.tm_q, q, 256, (uint64_t)(q_heads * seq), 128, kQT, true);
  for (int i = 0; i < 2; ++i) {
    enc = enc && encode_tma_rows(&a.tm_k[i], c.data[i], 256, (uint64_t)(G * c.capacity), 128, kKT, true);
    enc = enc && encode_tma_rows(&a.tm_v[i], c.data[2 + i], 256, (uint64_t)(G * c.capacity), 128, kKT, true);
  }
  MOTIF_REQUIRE(enc, MOTIF_ERR_CUDA, "prefill_attention: tensor map encoding failed");
  a.out = static_cast<__half*>(out);
  a.S = (int)seq;
  a.QH = (int)q_heads;
  a.cap = (int)c.capacity;
  a.off = (int)offset;
  a.off_dev = offset_dev;
  a.mode = mode;
  a.gr = (int)gr;
  a.q_origin = mode == 0 ? (int)(G * gr) : 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = err;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e =
        cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPASmem);
    if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "prefill_attention: smem attribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  // Split-KV for a single query tile over a long cache: up to one CTA per SM in total, at
  // least two key tiles per split.
  int nsplit = 1;
  const size_t ws_need = motif_prefill_attention_split_workspace_bytes(seq, q_heads);
  if (ws_need && workspace && workspace_bytes >= ws_need) {
    const int64_t nt_all = ceil_div(offset + seq, kKT);
    int64_t n = device_sms() / q_heads;
    if (n > nt_all / 2) n = nt_all / 2;
    if (n > kMaxSplits) n = kMaxSplits;
    if (n >= 2) nsplit = (int)n;
  }
  a.part = nsplit > 1 ? static_cast<float*>(workspace) : nullptr;
  cudaStream_t st = as_stream(stream);
  const dim3 grid((unsigned)ceil_div(seq, kQT), (unsigned)q_heads, (unsigned)nsplit);
  prefill_attn_kernel<<<grid, kPAThreads, kPASmem, st>>>(a);
  if (nsplit > 1) {
    const int rc = check_launch("prefill_attention");
    if (rc) return rc;
    prefill_merge_kernel<<<dim3((unsigned)seq, (unsigned)q_heads), 256, 0, st>>>(a.part, nsplit, (int)seq, (int)q_heads,
                                                                                 a.out);
    return check_launch("prefill_attention merge");
  }
  return check_launch("prefill_attention");
}
}  // namespace

extern "C" {

size_t motif_prefill_attention_split_workspace_bytes(int64_t seq, int64_t q_heads) {
  if (seq < 1 || seq > kQT || q_heads < 1 || q_heads > 65535) return 0;
  return sizeof(float) * kPartStride * (size_t)kMaxSplits * (size_t)q_heads * (size_t)seq;
}

int motif_prefill_attention(const void* q, int64_t seq, int64_t q_heads, const motif_kv4_slots* cache,
                            int64_t offset, int mode, int64_t gr, float scale, void* out, int* err, void* stream) {
  return prefill_attention(q, seq, q_heads, cache, offset, nullptr, mode, gr, scale, out, nullptr, 0, err, stream);
}

int motif_prefill_attention_split(const void* q, int64_t seq, int64_t q_heads, const motif_kv4_slots* cache,
                                  int64_t offset, const int32_t* offset_dev, int mode, int64_t gr, float scale,
                                  void* out, void* workspace, size_t workspace_bytes, int* err, void* stream) {
  return prefill_attention(q, seq, q_heads, cache, offset, offset_dev, mode, gr, scale, out, workspace,
                           workspace_bytes, err, stream);
}

int motif_prefill_post(const void* o, int64_t seq, int64_t q_heads, int mode, int64_t groups, int64_t gr,
                       const void* subln_w, const float* lambda_full, int64_t lambda_len, float lambda_init,
                       float eps, void* y, void* stream) {
  MOTIF_REQUIRE(o && subln_w && lambda_full && y, MOTIF_ERR_NULL, "prefill_post: null pointer");
  MOTIF_REQUIRE(mode == 0 || mode == 1, MOTIF_ERR_BAD_CONTRACT, "prefill_post: mode %d", mode);
  MOTIF_REQUIRE(seq >= 1 && seq < (1ll << 31) && groups >= 1 && groups < 65536, MOTIF_ERR_BAD_SHAPE,
                "prefill_post: seq=%lld groups=%lld", (long long)seq, (long long)groups);
  const int64_t want = mode == 0 ? groups * (gr + 1) : 2 * groups * gr;
  MOTIF_REQUIRE(q_heads == want, MOTIF_ERR_BAD_CONTRACT, "prefill_post: %lld heads, expected %lld",
                (long long)q_heads, (long long)want);
  int lam_mode = 0;
  if (mode == 0) {
    MOTIF_REQUIRE(lambda_len == 1 || lambda_len == groups || lambda_len == groups * gr, MOTIF_ERR_BAD_SHAPE,
                  "prefill_post: lambda_full has %lld values", (long long)lambda_len);
    lam_mode = lambda_len == 1 ? 0 : (lambda_len == groups ? 1 : 2);
  } else {
    MOTIF_REQUIRE(lambda_len == 1, MOTIF_ERR_BAD_SHAPE, "prefill_post: vanilla lambda is one value");
  }
  const dim3 grid((unsigned)seq, (unsigned)groups);
  const float out_scale = 1.0f - lambda_init;
  auto op = static_cast<const __half*>(o);
  auto wp = static_cast<const __half*>(subln_w);
  auto yp = static_cast<__half*>(y);
  cudaStream_t st = as_stream(stream);
  if (mode == 0)
    return launch_post<false>((int)gr, grid, st, op, (int)q_heads, (int)(groups * gr), wp, lambda_full, lam_mode,
                              out_scale, eps, yp);
  return launch_post<true>((int)gr, grid, st, op, (int)q_heads, 0, wp, lambda_full, 0, out_scale, eps, yp);
}

}  // extern "C"
