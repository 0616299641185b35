// Prefill GEMM on the 5th-generation tensor cores: Y[M, N] = X[M, K] · dequant(W)[N, K]^T with
// X fp16 row-major and W in the MLX affine q4 layout (group 64: uint32 words of eight nibbles,
// fp16 scale and bias per group). The prompt-length counterpart of the q4 GEMV: the reference
// runs every linear of a prompt through mx.quantized_matmul (nn.QuantizedLinear,
// src/mlx_motif/model.py:1047-1079), which dequantizes weight tiles to the activation type and
// multiplies them on the matrix units with fp32 accumulation; this kernel does the same on
// tcgen05.
//
// One CTA computes a 128 × BN (or 256 × BN: two row tiles sharing each dequantized B tile) tile
// of Y (BN 256 or 128) over K in 64-wide stages:
//   warp 0      one lane issues the TMA loads of a stage: the X tile (128 rows × 128 bytes in
//               the 128-byte swizzle, the tcgen05 K-major layout), the BN rows × 32 bytes of
//               packed codes and the BN × 16-byte boxes of scales and biases that hold the
//               stage's group.
//   warps 2..9  dequantize the codes (nibble -> fp16 by the 1024 + q exponent trick, then one
//               fused multiply-add with scale and bias) straight into the B tile, in the same
//               swizzled K-major layout, and signal the stage.
//   warp 1      owns the tensor memory (BN fp32 columns × 128 lanes); one lane issues four
//               tcgen05.mma (M 128, N BN, K 16) per stage and commits them to the stage's
//               "empty" barrier, which frees the stage for the next TMA round.
// After the last stage warps 2..9 read the accumulator back with tcgen05.ld (each warp the
// 32 TMEM lanes its index allows, half of the columns) and store fp16 rows.
//
// Every mbarrier wait is bounded. A wait that gives up raises the CTA's abort flag: the other
// roles leave their loops, the producer waits (bounded) for the loads it issued, the
// accumulator barrier still gets its commit, the tensor memory is freed, and the error word
// is set for the host to read.
#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace motif {
namespace {

constexpr int kGemmBM = 128;     // rows of X per CTA (the MMA's M)
constexpr int kDeqWarps = 8;     // dequantize + epilogue warps
constexpr int kGemmThreads = 32 * (2 + kDeqWarps);

struct GemmArgs {
  CUtensorMap tm_x;  // X as bytes: M rows × 2K bytes, box 128 × 128 B, 128-byte swizzle
  CUtensorMap tm_w;  // codes: N rows × K/2 bytes, box BN × 32 B
  CUtensorMap tm_s;  // scales: N rows × K/32 bytes, box BN × 16 B (8 groups)
  CUtensorMap tm_b;  // biases: same
  __half* y;
  const __half* residual;  // optional: y = fp16(fp16(X·Wᵀ) + residual), same layout as y
  int64_t M, N, K;
  int* err;  // optional error word (1 = a wait timed out)
};

template <int BN, int ST, int MT>
struct GemmLayout {
  static constexpr int kA = MT * kGemmBM * 128;  // X tiles (MT stacked 128-row tiles)
  static constexpr int kB = BN * 128;       // dequantized W tile
  static constexpr int kW = BN * 32;        // packed codes
  static constexpr int kS = BN * 16;        // scales (and biases) box
  static constexpr int kStage = kA + kB + kW + 2 * kS;
  static constexpr int kBars = ST * 3 + 1;
  static constexpr int kBytes = ST * kStage + kBars * 8 + 16 + 1024;  // + control words + alignment slack
  static_assert(kStage % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
};

__device__ __forceinline__ uint32_t dq_pair(uint32_t p, __half2 s2, __half2 b2) {
  const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));
  __half2 h = *reinterpret_cast<__half2*>(&p);
  h = __hfma2(__hsub2(h, k1024), s2, b2);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Eight nibbles (element e at bits 4e..4e+3) -> eight fp16 values in element order.
__device__ __forceinline__ uint4 dequant_word(uint32_t w, __half2 s2, __half2 b2) {
  const uint32_t t0 = (w & 0x000F000Fu) | 0x64006400u;          // (e0, e4)
  const uint32_t t1 = ((w >> 4) & 0x000F000Fu) | 0x64006400u;   // (e1, e5)
  const uint32_t t2 = ((w >> 8) & 0x000F000Fu) | 0x64006400u;   // (e2, e6)
  const uint32_t t3 = ((w >> 12) & 0x000F000Fu) | 0x64006400u;  // (e3, e7)
  uint4 o;
  o.x = dq_pair(__byte_perm(t0, t1, 0x5410), s2, b2);  // (e0, e1)
  o.y = dq_pair(__byte_perm(t2, t3, 0x5410), s2, b2);  // (e2, e3)
  o.z = dq_pair(__byte_perm(t0, t1, 0x7632), s2, b2);  // (e4, e5)
  o.w = dq_pair(__byte_perm(t2, t3, 0x7632), s2, b2);  // (e6, e7)
  return o;
}

// MT = 1 or 2 row tiles of 128 per CTA: with two, both MMAs of a K step read the same
// dequantized B tile, halving the dequant work per FLOP (accumulators: MT × BN TMEM columns).
template <int BN, int ST, int MT>
__global__ void __launch_bounds__(kGemmThreads, 1) q4_gemm_tc_kernel(const __grid_constant__ GemmArgs a) {
  using L = GemmLayout<BN, ST, MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST * L::kStage);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t sbase = tc::smem_addr(smem);
  const uint32_t bar0 = tc::smem_addr(bars);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto deq = [&](int s) { return bar0 + 8u * (ST + s); };
  auto empty = [&](int s) { return bar0 + 8u * (2 * ST + s); };
  const uint32_t acc = bar0 + 8u * (3 * ST);
  auto st_a = [&](int s) { return sbase + s * L::kStage; };
  auto st_b = [&](int s) { return sbase + s * L::kStage + L::kA; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)(a.K / 64);
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kGemmBM * MT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      tc::mbar_init(full(s), 1);
      tc::mbar_init(deq(s), kDeqWarps);
      tc::mbar_init(empty(s), 1);
    }
    tc::mbar_init(acc, 1);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_addr(tmem_slot), BN * MT);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer ----
      int issued = 0;
      for (int it = 0; it < nk; ++it) {
        const int s = it % ST;
        const uint32_t r = it / ST;
        if (it >= ST && !tc::mbar_wait(empty(s), (r - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const uint32_t base = st_a(s);
        tc::mbar_expect_tx(full(s), L::kA + L::kW + 2 * L::kS);
#pragma unroll
        for (int t = 0; t < MT; ++t) tc::tma_load_2d(base + t * 16384, &a.tm_x, it * 128, m0 + t * kGemmBM, full(s));
        tc::tma_load_2d(base + L::kA + L::kB, &a.tm_w, it * 32, n0, full(s));
        tc::tma_load_2d(base + L::kA + L::kB + L::kW, &a.tm_s, (it >> 3) * 16, n0, full(s));
        tc::tma_load_2d(base + L::kA + L::kB + L::kW + L::kS, &a.tm_b, (it >> 3) * 16, n0, full(s));
        issued = it + 1;
      }
      // every issued load lands before the CTA may exit (a no-op wait on the normal path)
      for (int it = issued > ST ? issued - ST : 0; it < issued; ++it)
        if (!tc::mbar_wait(full(it % ST), (it / ST) & 1)) *abort_flag = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer ----
      constexpr uint32_t idesc = tc::idesc_f16_f32(kGemmBM, BN);
      for (int it = 0; it < nk; ++it) {
        const int s = it % ST;
        const uint32_t par = (it / ST) & 1;
        if (!tc::mbar_wait(full(s), par) || !tc::mbar_wait(deq(s), par)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        tc::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t bdesc = tc::desc_kmajor_sw128(st_b(s) + kk * 32);
#pragma unroll
          for (int t = 0; t < MT; ++t)
            tc::mma_f16(tmem + t * BN, tc::desc_kmajor_sw128(st_a(s) + t * 16384 + kk * 32), bdesc, idesc,
                        (it | kk) != 0);
        }
        tc::mma_commit(empty(s));
      }
      tc::mma_commit(acc);  // also on abort: the accumulator barrier tracks the MMAs in flight
    }
    __syncwarp();
  } else {  // ---- dequantize, then the epilogue ----
    const int t = threadIdx.x - 64;
    constexpr int WPT = BN / 32;  // 32-bit code words per thread per stage
    const int flat = t * WPT, row = flat >> 3, w0 = flat & 7;
    for (int it = 0; it < nk; ++it) {
      const int s = it % ST;
      const bool landed = tc::mbar_wait(full(s), (it / ST) & 1);
      if (__any_sync(0xffffffffu, !landed || *abort_flag)) {  // warp-uniform exit
        if (!landed) *abort_flag = 1;
        break;
      }
      const uint8_t* stage = smem + s * L::kStage;
      const uint8_t* codes = stage + L::kA + L::kB + row * 32 + w0 * 4;
      const __half sc = *reinterpret_cast<const __half*>(stage + L::kA + L::kB + L::kW + row * 16 + (it & 7) * 2);
      const __half bi =
          *reinterpret_cast<const __half*>(stage + L::kA + L::kB + L::kW + L::kS + row * 16 + (it & 7) * 2);
      const __half2 s2 = __half2half2(sc), b2 = __half2half2(bi);
      uint32_t words[WPT];
#pragma unroll
      for (int j = 0; j < WPT; j += 4) {
        const uint4 v = *reinterpret_cast<const uint4*>(codes + j * 4);
        words[j] = v.x;
        words[j + 1] = v.y;
        words[j + 2] = v.z;
        words[j + 3] = v.w;
      }
      uint8_t* brow = smem + s * L::kStage + L::kA + row * 128;
#pragma unroll
      for (int j = 0; j < WPT; ++j) {
        const int c = w0 + j;  // 16-byte chunk of the 128-byte row
        *reinterpret_cast<uint4*>(brow + ((c ^ (row & 7)) << 4)) = dequant_word(words[j], s2, b2);
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(deq(s));
    }
    // epilogue: warp w reads TMEM lanes 32·(w mod 4) .. +31, columns [half·BN/2, (half+1)·BN/2)
    const bool ok = __all_sync(0xffffffffu, tc::mbar_wait(acc, 0));
    if (!ok) *abort_flag = 1;
    tc::tc_fence_after();
    const int q = warp & 3, half = (warp - 2) >> 2;
#pragma unroll 1
    for (int t = 0; t < MT; ++t) {
    const int64_t grow = m0 + t * kGemmBM + q * 32 + lane;
    const bool live = ok && !*abort_flag && grow < a.M;
#pragma unroll 1
    for (int cb = 0; cb < BN / 64; ++cb) {
      const int col = half * (BN / 2) + cb * 32;
      uint32_t r[32];
      tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + t * BN + col, r);
      tc::tmem_ld_wait();
      if (live) {
        __half* dst = a.y + grow * a.N + n0 + col;
        const __half* res = a.residual ? a.residual + grow * a.N + n0 + col : nullptr;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t o[4];
          uint4 rv = res ? *reinterpret_cast<const uint4*>(res + v * 8) : make_uint4(0, 0, 0, 0);
          const __half2* rh = reinterpret_cast<const __half2*>(&rv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __half2 h = __floats2half2_rn(__uint_as_float(r[v * 8 + 2 * e]), __uint_as_float(r[v * 8 + 2 * e + 1]));
            if (res) h = __hadd2(h, rh[e]);
            o[e] = *reinterpret_cast<uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(dst + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, BN * MT);
  }
  if (threadIdx.x == 0 && *abort_flag && a.err) atomicExch(a.err, 1);
}

template <int BN, int ST, int MT>
int launch_gemm(GemmArgs& a, cudaStream_t st) {
  using L = GemmLayout<BN, ST, MT>;
  auto kern = q4_gemm_tc_kernel<BN, ST, MT>;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "q4_gemm: smem attribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  const dim3 grid((unsigned)(a.N / BN), (unsigned)ceil_div(a.M, kGemmBM * MT));
  kern<<<grid, kGemmThreads, L::kBytes, st>>>(a);
  return check_launch("q4_gemm");
}

}  // namespace

bool q4_gemm_supported(int dtype, int bits, int group_size, int64_t m, int64_t n, int64_t k, const void* x,
                       const void* w, const void* sc, const void* bi, const void* y) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
  return dtype == MOTIF_F16 && bits == 4 && group_size == 64 && m >= kGemmBM && n % 128 == 0 && k % 512 == 0 &&
         k <= (1 << 20) && n <= (1 << 24) && al(x) && al(w) && al(sc) && al(bi) && al(y);
}

int q4_gemm(const void* x, int64_t m, int64_t k, const uint32_t* w, const void* scales, const void* biases, int64_t n,
            void* y, const void* residual, int* err, cudaStream_t st) {
  GemmArgs a{};
  const int bn = n % 256 == 0 ? 256 : 128;
  const bool enc = encode_tma_rows(&a.tm_x, x, (uint64_t)k * 2, (uint64_t)m, 128, kGemmBM, true) &&
                   encode_tma_rows(&a.tm_w, w, (uint64_t)k / 2, (uint64_t)n, 32, bn, false) &&
                   encode_tma_rows(&a.tm_s, scales, (uint64_t)k / 32, (uint64_t)n, 16, bn, false) &&
                   encode_tma_rows(&a.tm_b, biases, (uint64_t)k / 32, (uint64_t)n, 16, bn, false);
  MOTIF_REQUIRE(enc, MOTIF_ERR_CUDA, "q4_gemm: tensor map encoding failed");
  a.y = static_cast<__half*>(y);
  a.residual = static_cast<const __half*>(residual);
  a.M = m;
  a.N = n;
  a.K = k;
  a.err = err;
  // Two row tiles per CTA when the estimated time is lower: waves × per-CTA time, a two-tile CTA
  // taking about 1.6× a one-tile CTA (measured at 3204 × 28672 × 4096: 82 vs 51 µs per wave).
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  if (bn == 256) {
    const int64_t w1 = ceil_div((n / 256) * ceil_div(m, kGemmBM), sms);
    const int64_t w2 = ceil_div((n / 256) * ceil_div(m, 2 * kGemmBM), sms);
    if (16 * w2 < 10 * w1) return launch_gemm<256, 2, 2>(a, st);
  }
  return bn == 256 ? launch_gemm<256, 3, 1>(a, st) : launch_gemm<128, 4, 1>(a, st);
}

}  // namespace motif

extern "C" {

int motif_q4_gemm(const void* x, int64_t m, int64_t k, const uint32_t* w, const void* scales, const void* biases,
                  int64_t n, void* y, const void* residual, int* err, void* stream) {
  using namespace motif;
  MOTIF_REQUIRE(x && w && scales && biases && y, MOTIF_ERR_NULL, "q4_gemm: null pointer");
  MOTIF_REQUIRE(m > 0 && n > 0 && k > 0, MOTIF_ERR_BAD_SHAPE, "q4_gemm: m=%lld n=%lld k=%lld", (long long)m,
                (long long)n, (long long)k);
  MOTIF_REQUIRE(q4_gemm_supported(MOTIF_F16, 4, 64, m, n, k, x, w, scales, biases, y) &&
                    (!residual || reinterpret_cast<uintptr_t>(residual) % 16 == 0),
                MOTIF_ERR_BAD_CONTRACT,
                "q4_gemm: needs m >= 128, n %% 128 == 0, k %% 512 == 0 and 16-byte aligned operands "
                "(m=%lld n=%lld k=%lld)",
                (long long)m, (long long)n, (long long)k);
  return q4_gemm(x, m, k, w, scales, biases, n, y, residual, err, as_stream(stream));
}

}  // extern "C"
