// Affine-quantized linear y = x · dequant(W)ᵀ in the nn.QuantizedLinear
// layout (W (N, K·bits/32) uint32, scales/biases (N, K/g)).
//
// Decode fast path (bits 4, group 64, K % 128 == 0, fp16): HBM-streaming GEMV.
//   * A warp owns 16 output rows and a range of 512-wide K blocks. Each lane
//     streams 16-byte chunks of two rows (r, r+8) straight into registers,
//     double-buffered one block ahead.
//   * Nibbles become exact fp16 integers with the 0x6400 magic-exponent trick
//     (one LOP3 per nibble pair, one HSUB2/HFMA2 to remove the offset) and feed
//     mma.sync.m16n8k16 (fp16 × fp16 → fp32). The MMA is only a wide FMA here:
//     the kernel stays bound by HBM, and without it the per-nibble
//     convert+FMA work would make it issue-bound.
//   * The B operand's 8 columns are the 8 quantization groups of the block: a
//     lane feeds x only into the column of the group its k values belong to,
//     so column n accumulates Σ_{k∈g} x_k q_k for group g = 8·blk + n exactly
//     in fp32. Scales and biases are then applied per group in fp32:
//        y_n = Σ_g s_ng · dot_ng + b_ng · Σ_{k∈g} x_k
//     which is the affine quantized matmul formula (MLX qmv), not a
//     dequantize-to-fp16 approximation.
//   * x is staged once per CTA in shared memory, permuted to the nibble order
//     the dequant produces, with per-group sums of x.
//   * Split-K writes fp32 partials that a small kernel (or the consumer) sums.
//
// General path (bits 4/8, group 32/64/128, any K % 32 == 0): CUDA-core GEMV,
// one warp per output row, exact fp32 per-nibble MACs. Used for shapes the
// fast path does not cover.
#include "common.cuh"

namespace motif {
namespace {

// (a & b) | c in one instruction.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Word of 8 nibbles n0..n7 -> four f16x2 registers (n0,n4) (n1,n5) (n2,n6) (n3,n7).
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t LO = 0x000F000Fu, HI = 0x00F000F0u, EX = 0x64006400u;
  const uint32_t t0 = lop3_and_or(w, LO, EX);
  const uint32_t t1 = lop3_and_or(w, HI, EX);
  const uint32_t w8 = w >> 8;
  const uint32_t t2 = lop3_and_or(w8, LO, EX);
  const uint32_t t3 = lop3_and_or(w8, HI, EX);
  const uint32_t k1024 = 0x64006400u;  // {1024, 1024}
  const uint32_t k1_16 = 0x2C002C00u;  // {1/16, 1/16}
  const uint32_t km64 = 0xD400D400u;   // {-64, -64}
  asm("sub.f16x2 %0, %1, %2;\n" : "=r"(p[0]) : "r"(t0), "r"(k1024));
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(p[1]) : "r"(t1), "r"(k1_16), "r"(km64));
  asm("sub.f16x2 %0, %1, %2;\n" : "=r"(p[2]) : "r"(t2), "r"(k1024));
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(p[3]) : "r"(t3), "r"(k1_16), "r"(km64));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kRowsPerWarp = 16;
constexpr int kRowsPerCta = kGemvWarps * kRowsPerWarp;  // 64
constexpr int kBlockK = 512;

struct BlockRegs {
  uint4 wr[4];   // row r:   chunk q (32 nibbles) of this block
  uint4 wr8[4];  // row r+8
  uint32_t s, s8, b, b8;  // half2 scales / biases of groups (g0, g0+1), rows r and r+8
};

__device__ __forceinline__ void load_block(BlockRegs& R, const uint32_t* __restrict__ w,
                                           const __half* __restrict__ sc,
                                           const __half* __restrict__ bi, int64_t row_r,
                                           int64_t row_r8, int64_t wpr, int64_t gpr, int blk,
                                           int quarters, int c) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q < quarters) {
      const int64_t word = (int64_t)blk * 64 + q * 16 + c * 4;
      R.wr[q] = __ldg(reinterpret_cast<const uint4*>(w + row_r * wpr + word));
      R.wr8[q] = __ldg(reinterpret_cast<const uint4*>(w + row_r8 * wpr + word));
    }
  }
  const int64_t g0 = (int64_t)blk * 8 + 2 * c;
  if (g0 < gpr) {
    R.s = __ldg(reinterpret_cast<const uint32_t*>(sc + row_r * gpr + g0));
    R.s8 = __ldg(reinterpret_cast<const uint32_t*>(sc + row_r8 * gpr + g0));
    R.b = __ldg(reinterpret_cast<const uint32_t*>(bi + row_r * gpr + g0));
    R.b8 = __ldg(reinterpret_cast<const uint32_t*>(bi + row_r8 * gpr + g0));
  }
}

__device__ __forceinline__ float2 h2f(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// One 512-wide K block of one warp: 32 MMAs, then the per-group affine epilogue.
__device__ __forceinline__ void compute_block(const BlockRegs& R, const __half* __restrict__ xp_s,
                                              const float* __restrict__ xsum_s, int blk, int blk0,
                                              int quarters, int64_t gpr, int c, int q_lane,
                                              float& acc_r, float& acc_r8) {
  // This lane's x chunk (permuted fp16): only needed by lanes whose quarter exists.
  uint32_t xr[16];
  if (q_lane >= 0 && q_lane < quarters) {
    const uint4* src = reinterpret_cast<const uint4*>(xp_s + (blk - blk0) * kBlockK + q_lane * 128 + c * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 v = src[i];
      xr[4 * i + 0] = v.x;
      xr[4 * i + 1] = v.y;
      xr[4 * i + 2] = v.z;
      xr[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) xr[i] = 0u;
  }
  float C[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q >= quarters) break;
    const bool mine = (q == q_lane);
    const uint32_t wrq[4] = {R.wr[q].x, R.wr[q].y, R.wr[q].z, R.wr[q].w};
    const uint32_t wr8q[4] = {R.wr8[q].x, R.wr8[q].y, R.wr8[q].z, R.wr8[q].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t P[4], P8[4];
      dequant_word(wrq[j], P);
      dequant_word(wr8q[j], P8);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t b0 = mine ? xr[4 * j + 2 * h] : 0u;
        const uint32_t b1 = mine ? xr[4 * j + 2 * h + 1] : 0u;
        mma16816(C, P[2 * h], P8[2 * h], P[2 * h + 1], P8[2 * h + 1], b0, b1);
      }
    }
  }
  const int64_t g0 = (int64_t)blk * 8 + 2 * c;
  if (g0 < gpr) {
    const int lg = (int)(g0 - (int64_t)blk0 * 8);
    const float xs0 = xsum_s[lg], xs1 = xsum_s[lg + 1];
    const float2 s = h2f(R.s), s8 = h2f(R.s8), b = h2f(R.b), b8 = h2f(R.b8);
    acc_r += s.x * C[0] + s.y * C[1] + b.x * xs0 + b.y * xs1;
    acc_r8 += s8.x * C[2] + s8.y * C[3] + b8.x * xs0 + b8.y * xs1;
  }
}

// grid (ceil(N / 64), ksplit); dynamic smem: permuted x of the CTA's K range + group sums.
__global__ void __launch_bounds__(kGemvThreads) q4_gemv_mma_kernel(
    const __half* __restrict__ x, int64_t K, const uint32_t* __restrict__ w,
    const __half* __restrict__ sc, const __half* __restrict__ bi, int64_t N, int blocks_per_split,
    __half* __restrict__ y, float* __restrict__ partial) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int nblk = (int)((K + kBlockK - 1) / kBlockK);
  const int blk0 = blockIdx.y * blocks_per_split;
  const int blk1 = min(nblk, blk0 + blocks_per_split);
  const int64_t k0 = (int64_t)blk0 * kBlockK;
  const int64_t k1 = min(K, (int64_t)blk1 * kBlockK);
  const int64_t klen = k1 - k0;  // multiple of 128
  __half* xp_s = reinterpret_cast<__half*>(smem_raw);
  float* xsum_s = reinterpret_cast<float*>(smem_raw + (size_t)blocks_per_split * kBlockK * sizeof(__half));

  // ---- stage x: permute each 8-value word to (x0,x4,x1,x5,x2,x6,x3,x7); group sums ----
  for (int64_t wi = threadIdx.x; wi < klen / 8; wi += kGemvThreads) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + k0 + wi * 8);
    const __half* e = reinterpret_cast<const __half*>(&v);
    uint4 o;
    __half* oe = reinterpret_cast<__half*>(&o);
    oe[0] = e[0]; oe[1] = e[4]; oe[2] = e[1]; oe[3] = e[5];
    oe[4] = e[2]; oe[5] = e[6]; oe[6] = e[3]; oe[7] = e[7];
    *reinterpret_cast<uint4*>(xp_s + wi * 8) = o;
  }
  for (int64_t g = threadIdx.x; g < klen / 64; g += kGemvThreads) {
    const uint4* src = reinterpret_cast<const uint4*>(x + k0 + g * 64);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 v = src[i];
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __half22float2(h[t]);
        s += f.x + f.y;
      }
    }
    xsum_s[g] = s;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int64_t tile_row = (int64_t)blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
  if (tile_row >= N) return;
  const int64_t row_r = min(tile_row + r, N - 1);
  const int64_t row_r8 = min(tile_row + r + 8, N - 1);
  const int64_t wpr = K / 8, gpr = K / 64;
  // The quarter whose group feeds this lane's B column (column r = group 2q + c/2).
  const int diff = r - (c >> 1);
  const int q_lane = (diff >= 0 && (diff & 1) == 0) ? diff >> 1 : -1;

  float acc_r = 0.f, acc_r8 = 0.f;
  auto quarters_of = [&](int blk) -> int {
    const int64_t rem = K - (int64_t)blk * kBlockK;
    return rem >= kBlockK ? 4 : (int)(rem / 128);
  };
  BlockRegs A, B;
  if (blk0 < blk1) load_block(A, w, sc, bi, row_r, row_r8, wpr, gpr, blk0, quarters_of(blk0), c);
  for (int blk = blk0; blk < blk1; blk += 2) {
    const bool has1 = blk + 1 < blk1;
    if (has1) load_block(B, w, sc, bi, row_r, row_r8, wpr, gpr, blk + 1, quarters_of(blk + 1), c);
    compute_block(A, xp_s, xsum_s, blk, blk0, quarters_of(blk), gpr, c, q_lane, acc_r, acc_r8);
    if (has1) {
      if (blk + 2 < blk1) load_block(A, w, sc, bi, row_r, row_r8, wpr, gpr, blk + 2, quarters_of(blk + 2), c);
      compute_block(B, xp_s, xsum_s, blk + 1, blk0, quarters_of(blk + 1), gpr, c, q_lane, acc_r, acc_r8);
    }
  }
  acc_r += __shfl_xor_sync(0xffffffffu, acc_r, 1);
  acc_r += __shfl_xor_sync(0xffffffffu, acc_r, 2);
  acc_r8 += __shfl_xor_sync(0xffffffffu, acc_r8, 1);
  acc_r8 += __shfl_xor_sync(0xffffffffu, acc_r8, 2);
  if (c == 0) {
    const int64_t n_r = tile_row + r, n_r8 = tile_row + r + 8;
    if (partial) {
      float* p = partial + (int64_t)blockIdx.y * N;
      if (n_r < N) p[n_r] = acc_r;
      if (n_r8 < N) p[n_r8] = acc_r8;
    } else {
      if (n_r < N) y[n_r] = __float2half_rn(acc_r);
      if (n_r8 < N) y[n_r8] = __float2half_rn(acc_r8);
    }
  }
}

__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int ksplit, int64_t N,
                                     __half* __restrict__ y) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float s = 0.f;
  for (int i = 0; i < ksplit; ++i) s += partial[(int64_t)i * N + n];
  y[n] = __float2half_rn(s);
}

// ---- general CUDA-core path: one warp per (row, m) --------------------------
template <typename T>
__global__ void qlinear_general_kernel(const T* __restrict__ x, int64_t M, int64_t K,
                                       const uint32_t* __restrict__ w, const T* __restrict__ sc,
                                       const T* __restrict__ bi, int64_t N, int bits, int gs,
                                       T* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t idx = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (idx >= M * N) return;
  const int64_t m = idx / N, n = idx - (idx / N) * N;
  const int el = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  const int64_t wpr = K / el, gpr = K / gs;
  const T* xm = x + m * K;
  float acc = 0.f;
  for (int64_t wi = lane; wi < wpr; wi += 32) {
    const uint32_t word = w[n * wpr + wi];
    const int64_t k0 = wi * el;
    const int64_t g = k0 / gs;
    const float s = to_f<T>(sc[n * gpr + g]);
    const float b = to_f<T>(bi[n * gpr + g]);
    float dot = 0.f, xs = 0.f;
    for (int j = 0; j < el; ++j) {
      const float xv = to_f<T>(xm[k0 + j]);
      dot += xv * (float)((word >> (j * bits)) & mask);
      xs += xv;
    }
    acc += s * dot + b * xs;
  }
  acc = warp_sum(acc);
  if (lane == 0) y[m * N + n] = from_f<T>(acc);
}

struct GemvPlan {
  int ksplit;
  int blocks_per_split;
  size_t smem;
};

GemvPlan plan_gemv(int64_t N, int64_t K) {
  const int nblk = (int)ceil_div(K, kBlockK);
  const int64_t ctas_n = ceil_div(N, kRowsPerCta);
  // Enough CTAs to keep ~8 per SM streaming; at least 2 blocks (1024 K) per split.
  int64_t want = ceil_div(148 * 8, ctas_n);
  int64_t max_by_k = nblk / 2 > 0 ? nblk / 2 : 1;
  int64_t ks = want < max_by_k ? want : max_by_k;
  if (ks < 1) ks = 1;
  int bps = (int)ceil_div(nblk, ks);
  ks = ceil_div(nblk, bps);
  GemvPlan p;
  p.ksplit = (int)ks;
  p.blocks_per_split = bps;
  p.smem = (size_t)bps * kBlockK * sizeof(__half) + (size_t)bps * 8 * sizeof(float);
  return p;
}

bool fast_path_ok(int dtype, int bits, int gs, int64_t K, const void* x, const void* w,
                  const void* sc, const void* bi) {
  auto a = [](const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
  return dtype == MOTIF_F16 && bits == 4 && gs == 64 && K % 128 == 0 && K <= (1 << 20) &&
         a(x, 16) && a(w, 16) && a(sc, 4) && a(bi, 4);
}

}  // namespace
}  // namespace motif

using namespace motif;

extern "C" {

size_t motif_quantized_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int bits,
                                              int group_size) {
  if (bits != 4 || group_size != 64 || k % 128 != 0) return 0;
  GemvPlan p = plan_gemv(n, k);
  return p.ksplit > 1 ? sizeof(float) * (size_t)p.ksplit * (size_t)n * (size_t)(m > 0 ? 1 : 0) : 0;
}

int motif_quantized_linear(int dtype, int bits, int group_size, const void* x, int64_t m,
                           int64_t k, const uint32_t* w, const void* scales, const void* biases,
                           int64_t n, void* y, void* workspace, size_t workspace_bytes,
                           void* stream) {
  MOTIF_REQUIRE(x && w && scales && biases && y, MOTIF_ERR_NULL, "quantized_linear: null pointer");
  MOTIF_REQUIRE(bits == 4 || bits == 8, MOTIF_ERR_DTYPE, "quantized_linear: bits=%d not in {4,8}", bits);
  MOTIF_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, MOTIF_ERR_BAD_CONTRACT,
                "quantized_linear: group_size=%d not in {32,64,128}", group_size);
  MOTIF_REQUIRE(m >= 0 && n > 0 && k > 0 && k % group_size == 0 && k % 32 == 0, MOTIF_ERR_BAD_SHAPE,
                "quantized_linear: m=%lld n=%lld k=%lld", (long long)m, (long long)n, (long long)k);
  if (m == 0) return MOTIF_OK;
  cudaStream_t st = as_stream(stream);
  if (fast_path_ok(dtype, bits, group_size, k, x, w, scales, biases)) {
    GemvPlan p = plan_gemv(n, k);
    float* part = nullptr;
    if (p.ksplit > 1) {
      const size_t need = sizeof(float) * (size_t)p.ksplit * (size_t)n;
      if (!workspace || workspace_bytes < need) {
        // No (or short) workspace: run unsplit.
        p.ksplit = 1;
        p.blocks_per_split = (int)ceil_div(k, kBlockK);
        p.smem = (size_t)p.blocks_per_split * kBlockK * sizeof(__half) + (size_t)p.blocks_per_split * 8 * sizeof(float);
      } else {
        part = static_cast<float*>(workspace);
      }
    }
    static bool configured = false;
    if (!configured) {
      cudaError_t e = cudaFuncSetAttribute(q4_gemv_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "quantized_linear: smem attribute: %s", cudaGetErrorString(e));
      configured = true;
    }
    MOTIF_REQUIRE(p.smem <= 200 * 1024, MOTIF_ERR_BAD_SHAPE, "quantized_linear: K=%lld too large", (long long)k);
    dim3 grid((unsigned)ceil_div(n, kRowsPerCta), p.ksplit);
    for (int64_t i = 0; i < m; ++i) {
      const __half* xi = static_cast<const __half*>(x) + i * k;
      __half* yi = static_cast<__half*>(y) + i * n;
      q4_gemv_mma_kernel<<<grid, kGemvThreads, p.smem, st>>>(
          xi, k, w, static_cast<const __half*>(scales), static_cast<const __half*>(biases), n,
          p.blocks_per_split, yi, part);
      if (part) splitk_reduce_kernel<<<ceil_div(n, 256), 256, 0, st>>>(part, p.ksplit, n, yi);
    }
    return check_launch("quantized_linear (mma)");
  }
  const int warps = 8;
  const int64_t blocks = ceil_div(m * n, warps);
  MOTIF_DISPATCH_FLOAT(dtype, T, {
    qlinear_general_kernel<T><<<blocks, warps * 32, 0, st>>>(
        static_cast<const T*>(x), m, k, w, static_cast<const T*>(scales),
        static_cast<const T*>(biases), n, bits, group_size, static_cast<T*>(y));
  });
  return check_launch("quantized_linear (general)");
}

}  // extern "C"
