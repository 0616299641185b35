// Affine-quantized linear y = x · dequant(W)ᵀ in the nn.QuantizedLinear
// layout (W (N, K·bits/32) uint32, scales/biases (N, K/g)).
//
// Decode fast path (bits 4, group 64, K % 128 == 0, fp16): a persistent
// HBM-streaming GEMV.
//   * Work unit = (16-row tile, 512-wide K block). Units are ordered tile-major
//     and every warp of the grid takes one contiguous run of them (stream-K),
//     so all warps stream the same number of bytes whatever N and K are.
//   * A lane streams 16-byte chunks of its two rows (r, r+8) straight into
//     registers, one unit ahead of the one it computes. The first unit's loads
//     are issued before `griddepcontrol.wait`: launched with programmatic
//     stream serialization, the kernel's weight stream starts while the
//     previous kernel is still finishing, and only reading x waits for it.
//   * Nibbles become exact fp16 integers with the 0x6400 magic exponent (one
//     LOP3 per nibble pair, one HSUB2/HFMA2 to drop the offset) and feed
//     mma.sync.m16n8k16 (fp16 × fp16 → fp32). The MMA is a wide FMA: without
//     it the per-nibble convert+FMA work would make the kernel issue-bound.
//   * The B operand's 8 columns are the 8 quantization groups of a K block:
//     a lane feeds x only into the column of the group its k values belong
//     to, so column n accumulates Σ_{k∈g} x_k q_k for group g = 8·blk + n
//     exactly in fp32, and the affine epilogue y = Σ_g s·dot + b·Σx runs in
//     fp32 (the MLX quantized-matmul formula).
//   * A tile split across warps is finished by the last contributing warp:
//     partials go to the workspace, an atomic counter per tile elects the
//     last warp (no waiting), which sums the partials in slot order
//     (deterministic), writes fp16 and resets the counter to zero.
//   * x is staged once per CTA in shared memory, permuted to the nibble order
//     the dequant produces, with per-group sums. Optional prologues build x
//     in place: rms_norm(h + delta)·w (residual + norm, optionally gathering
//     h from the embedding table), or polynorm(gate)·up from per-tile
//     (Σg², Σg⁴, Σg⁶) statistics. An optional epilogue writes those
//     statistics for output rows [0, stats_rows) (the gate half of a fused
//     gate|up projection).
//
// General path (bits 4/8, group 32/64/128, any K % 32 == 0): CUDA-core GEMV,
// one warp per output row, exact fp32 per-nibble MACs. Used for shapes the
// fast path does not cover.
#include <cuda.h>

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

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;\n"); }

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kBlockK = 512;
constexpr int kTileRows = 16;
// Staged x of the TMA kernel: each 64-value group takes 144 B (16 B of padding), so the
// quad-diagonal lanes, which read four groups at the same offset, land on distinct banks.
constexpr int kXGroupBytes = 144;
// Zeros read by the lanes that feed no B column: covers groups c and c+4 (4·144 + 128 B).
constexpr int kZeroBytes = 768;
// Workspace layout: [tile counters: kCounterTiles int32][split-K partials]. The
// counter region has a fixed size so that GEMVs of different shapes can share
// one workspace: partials of one shape never land on another shape's counters.
constexpr int64_t kCounterTiles = 16384;
constexpr size_t kCounterBytes = sizeof(int) * kCounterTiles;
// Control words at the top of the counter region: [kCounterTiles-1] error word,
// [kCounterTiles-2] argmax tiles finished, [kCounterTiles-4 .. -3] argmax key (8-byte aligned).
constexpr int64_t kErrSlot = kCounterTiles - 1;
constexpr int64_t kAmaxTilesSlot = kCounterTiles - 2;
constexpr int64_t kAmaxKeySlot = kCounterTiles - 4;
constexpr int64_t kTpWaitSlot = kCounterTiles - 8;     // [-8 .. -7] exchange-read time, ns (int64)
constexpr int64_t kTileCounterCap = kCounterTiles - 8;  // split-tile counters: N up to 262016 rows

enum : int { kModeX = 0, kModeAddRms = 1, kModePoly = 2 };

struct LinArgs {
  // TMA descriptors of the weight codes, scales and biases (TMA kernel only).
  alignas(64) CUtensorMap tm_w;
  alignas(64) CUtensorMap tm_s;
  alignas(64) CUtensorMap tm_b;
  int* err;  // set non-zero if a TMA wait ran out (the kernel then stops early)
  const uint32_t* w;
  const __half* sc;
  const __half* bi;
  int64_t N, K;
  int nblk, ntiles;
  int64_t units;
  int total_warps;
  __half* y;
  float* partial;  // multi-row kernel: [ntiles][maxc][16 * rows] floats
  long long* ppair;  // one-row kernels: [ntiles][maxc][16] (value, 1) pairs, zero between calls
  int* counters;   // [ntiles], zero between calls (multi-row kernel)
  int maxc;
  // prologue
  int mode;
  const __half* x;
  const __half* h_in;
  const int32_t* token;
  const __half* embed;
  int64_t vocab;
  const __half* delta;
  __half* h_out;
  const __half* norm_w;
  float eps;
  const __half* gate;
  const __half* up;
  const float* stats;
  int stats_count;
  const __half* poly_w;
  const __half* poly_b;
  float poly_eps;
  float poly_inv_dim;
  // epilogue
  float* stats_out;
  int64_t stats_rows;
  // fused greedy argmax over the outputs (optional)
  unsigned long long* amax_key;  // packed (ordered value, inverted index), 0 between calls
  int* amax_tiles;               // finished tiles, 0 between calls
  int32_t* argmax_out;
  int32_t* pos_len_inc;
  long long* argmax_key_out;
  int64_t argmax_row_offset;
  // tensor-parallel exchange over peer memory (tp_world 0: none); values travel as
  // (fp32 bits, number) pairs, one 8-byte store each
  int tp_world;
  const int* tp_seq;
  int tp_tag;
  long long* tp_out[8];
  long long* tp_stats[8];
  const long long* tp_in;
  const long long* tp_stats_in;
  unsigned long long* tp_wait_ns;  // CTA 0 adds the time its exchange reads took (tp_world > 0)
};

constexpr unsigned long long kTpWaitNs = 2000ull * 1000 * 1000;  // exchange wait limit (2 s)

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int tp_number(const LinArgs& a) { return (*a.tp_seq + 1) * 1024 + a.tp_tag; }

__device__ __forceinline__ long long tp_pair(float v, int number) {
  return (long long)(((unsigned long long)(uint32_t)number << 32) | __float_as_uint(v));
}

// Exchange accesses. A pair is one naturally aligned 64-bit element, stored and loaded as a
// single relaxed system-scope access (peers write it over NVLink), so a reader that sees the
// expected number also sees the value stored with it: a pair cannot tear, and no fence is
// needed because nothing else is read on the strength of it.
__device__ __forceinline__ void tp_store(long long* p, long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ long long tp_load(const long long* p) {
  long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Two adjacent pairs in one 16-byte load; each 64-bit element is its own single-copy-atomic
// access (the vector form does not make the two elements one access, nor does it need to).
__device__ __forceinline__ void tp_load2(const long long* p, long long& a, long long& b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];\n" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Read an exchanged pair written by some rank, re-reading until it carries `number`; on
// time-out it records the error and returns what is there.
__device__ __forceinline__ float tp_read(const long long* p, int number, int* err) {
  long long x = tp_load(p);
  if ((int)(x >> 32) != number) {
    const unsigned long long t0 = global_ns();
    do {
      __nanosleep(32);
      x = tp_load(p);
      if (global_ns() - t0 > kTpWaitNs) {
        if (err) atomicExch(err, 2);
        break;
      }
    } while ((int)(x >> 32) != number);
  }
  return __uint_as_float((uint32_t)x);
}

// Split-tile partials of the one-row kernels. A warp that shares a tile with others stores
// its 16 row sums as 8-byte (fp32 value, kPartMark) pairs and moves on — no fence, no counter, no
// round trip. The tile's first warp (slot 0), whose range ends with the tile and which
// therefore finishes it last, keeps its own sums in registers, reads the other slots until
// each carries the marker, adds them in slot order and clears them (the region is zero
// between launches). Each pair is one naturally aligned 64-bit access, so a reader that sees
// the marker sees the value stored with it. The waits point only at warps of higher index,
// which never wait on lower ones, and the grid is at most one CTA per SM, so every wait
// ends; a wait that still runs out (200 ms) sets the error word.
constexpr unsigned long long kPartWaitNs = 200ull * 1000 * 1000;
// The marker word: a NaN pattern that no arithmetic produces (CUDA's NaN results are
// 0x7FFFFFFF), so a float left in the region by some other use cannot pass for it.
constexpr uint32_t kPartMark = 0x7FF0A001u;

__device__ __forceinline__ void part_store(long long* p, float v) {
  const long long q = (long long)(((unsigned long long)kPartMark << 32) | __float_as_uint(v));
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;\n" ::"l"(p), "l"(q) : "memory");
}

__device__ __forceinline__ long long part_load(const long long* p) {
  long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// s (slot 0's sum) + slots 1..nc-1 of one row, in slot order. The loads of kChunk slots go out
// together; slots not yet carrying the marker are re-read together until all do (bounded).
template <int kChunk>
__device__ __forceinline__ float part_reduce(long long* p, int nc, float s, int* err) {
  for (int i0 = 1; i0 < nc; i0 += kChunk) {
    long long q[kChunk];
    uint32_t pending = 0;
#pragma unroll
    for (int j = 0; j < kChunk; ++j)
      if (i0 + j < nc) q[j] = part_load(p + (int64_t)(i0 + j) * kTileRows);
#pragma unroll
    for (int j = 0; j < kChunk; ++j)
      if (i0 + j < nc && (uint32_t)((unsigned long long)q[j] >> 32) != kPartMark) pending |= 1u << j;
    if (pending) {
      const unsigned long long t0 = global_ns();
      while (pending) {
#pragma unroll
        for (int j = 0; j < kChunk; ++j)
          if (pending & (1u << j)) q[j] = part_load(p + (int64_t)(i0 + j) * kTileRows);
#pragma unroll
        for (int j = 0; j < kChunk; ++j)
          if ((pending & (1u << j)) && (uint32_t)((unsigned long long)q[j] >> 32) == kPartMark) pending &= ~(1u << j);
        if (pending && global_ns() - t0 > kPartWaitNs) {
          if (err) atomicExch(err, 3);
          break;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      if (i0 + j < nc) {
        s += __uint_as_float((uint32_t)q[j]);
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;\n" ::"l"(p + (int64_t)(i0 + j) * kTileRows), "l"(0ll)
                     : "memory");
      }
    }
  }
  return s;
}

struct UnitRegs {
  uint4 wr[4];
  uint4 wr8[4];
  uint32_t s, s8, b, b8;
};

__device__ __forceinline__ int quarters_of(const LinArgs& a, int blk) {
  const int64_t rem = a.K - (int64_t)blk * kBlockK;
  return rem >= kBlockK ? 4 : (int)(rem / 128);
}

__device__ __forceinline__ void load_unit(UnitRegs& R, const LinArgs& a, int tile, int blk, int r, int c) {
  const int64_t row_r = min((int64_t)tile * kTileRows + r, a.N - 1);
  const int64_t row_r8 = min((int64_t)tile * kTileRows + r + 8, a.N - 1);
  const int64_t wpr = a.K / 8, gpr = a.K / 64;
  const int quarters = quarters_of(a, blk);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q < quarters) {
      const int64_t word = (int64_t)blk * 64 + q * 16 + c * 4;
      R.wr[q] = __ldg(reinterpret_cast<const uint4*>(a.w + row_r * wpr + word));
      R.wr8[q] = __ldg(reinterpret_cast<const uint4*>(a.w + row_r8 * wpr + word));
    }
  }
  const int64_t g0 = (int64_t)blk * 8 + 2 * c;
  if (g0 < gpr) {
    R.s = __ldg(reinterpret_cast<const uint32_t*>(a.sc + row_r * gpr + g0));
    R.s8 = __ldg(reinterpret_cast<const uint32_t*>(a.sc + row_r8 * gpr + g0));
    R.b = __ldg(reinterpret_cast<const uint32_t*>(a.bi + row_r * gpr + g0));
    R.b8 = __ldg(reinterpret_cast<const uint32_t*>(a.bi + row_r8 * gpr + g0));
  }
}

__device__ __forceinline__ float2 h2f(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// One unit: 32 MMAs over a 512-wide K block, then the per-group affine epilogue.
__device__ __forceinline__ void compute_unit(const UnitRegs& R, const LinArgs& a, int blk,
                                             const __half* __restrict__ xp_s,
                                             const float* __restrict__ xsum_s, int c, int q_lane,
                                             float& acc_r, float& acc_r8) {
  const int quarters = quarters_of(a, blk);
  uint32_t xr[16];
  if (q_lane >= 0 && q_lane < quarters) {
    const uint4* src = reinterpret_cast<const uint4*>(xp_s + (int64_t)blk * kBlockK + q_lane * 128 + c * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = src[i];
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
  if (g0 < a.K / 64) {
    const float xs0 = xsum_s[g0], xs1 = xsum_s[g0 + 1];
    const float2 s = h2f(R.s), s8 = h2f(R.s8), b = h2f(R.b), b8 = h2f(R.b8);
    acc_r += s.x * C[0] + s.y * C[1] + b.x * xs0 + b.y * xs1;
    acc_r8 += s8.x * C[2] + s8.y * C[3] + b8.x * xs0 + b8.y * xs1;
  }
}

// The warp whose unit range [u·W/U, (u+1)·W/U) contains unit u (32-bit: the host
// guarantees units · total_warps < 2^32).
__device__ __forceinline__ int warp_of_unit(uint32_t u, uint32_t units, uint32_t tw) {
  return (int)(((u + 1) * tw - 1) / units);
}

// Finish this warp's share of a tile: write it, or publish a partial (the tile's first warp
// reduces, see part_store). Also emits the tile's PolyNorm statistics when asked.
template <int kChunk>
__device__ void tile_epilogue(const LinArgs& a, int tile, int gw, float acc_r, float acc_r8, int lane) {
  const int r = lane >> 2, c = lane & 3;
  acc_r += __shfl_xor_sync(0xffffffffu, acc_r, 1);
  acc_r += __shfl_xor_sync(0xffffffffu, acc_r, 2);
  acc_r8 += __shfl_xor_sync(0xffffffffu, acc_r8, 1);
  acc_r8 += __shfl_xor_sync(0xffffffffu, acc_r8, 2);
  const uint32_t u_first = (uint32_t)tile * (uint32_t)a.nblk;
  const int w_first = warp_of_unit(u_first, (uint32_t)a.units, (uint32_t)a.total_warps);
  const int w_last = warp_of_unit(u_first + a.nblk - 1, (uint32_t)a.units, (uint32_t)a.total_warps);
  const int nc = w_last - w_first + 1;
  const int64_t row0 = (int64_t)tile * kTileRows;
  // Final fp16 values of this tile's rows, held by lanes 0..15 (row = row0 + lane).
  float v = 0.f;
  bool have = false;
  if (nc == 1) {
    // Gather rows r / r+8 from the c == 0 lanes into lanes 0..15.
    const float a_r = __shfl_sync(0xffffffffu, acc_r, (lane & 7) * 4);
    const float a_r8 = __shfl_sync(0xffffffffu, acc_r8, (lane & 7) * 4);
    v = lane < 8 ? a_r : a_r8;
    have = lane < kTileRows;
  } else {
    const int slot = gw - w_first;
    long long* p = a.ppair + (int64_t)tile * a.maxc * kTileRows;
    if (slot > 0) {
      if (c == 0) {
        part_store(p + slot * kTileRows + r, acc_r);
        part_store(p + slot * kTileRows + r + 8, acc_r8);
      }
    } else {
      const float a_r = __shfl_sync(0xffffffffu, acc_r, (lane & 7) * 4);
      const float a_r8 = __shfl_sync(0xffffffffu, acc_r8, (lane & 7) * 4);
      if (lane < kTileRows) {
        float s = 0.f;
        s += lane < 8 ? a_r : a_r8;  // slot 0: this warp's sums
        v = part_reduce<kChunk>(p + lane, nc, s, a.err);
        have = true;
      }
    }
  }
  const int64_t row = row0 + lane;
  const __half hv = __float2half_rn(v);
  if (have && row < a.N) {
    a.y[row] = hv;
    if (a.tp_world && a.tp_out[0]) {  // this rank's fp32 rows into every rank's exchange buffer
      const long long pr = tp_pair(v, tp_number(a));
      for (int r = 0; r < a.tp_world; ++r) tp_store(a.tp_out[r] + row, pr);
    }
  }
  // all-or-nothing per warp: `have` is uniform across lanes 0..15 of the finishing warp
  const bool any = __any_sync(0xffffffffu, have);
  if (any && (a.stats_out || (a.tp_world && a.tp_stats[0])) && row0 < a.stats_rows) {
    const float f = (have && row < a.stats_rows) ? __half2float(hv) : 0.f;
    const float f2 = f * f, f4 = f2 * f2;
    float s2 = warp_sum(f2), s4 = warp_sum(f4), s6 = warp_sum(f4 * f2);
    if (lane == 0) {
      if (a.stats_out) {
        a.stats_out[tile * 3 + 0] = s2;
        a.stats_out[tile * 3 + 1] = s4;
        a.stats_out[tile * 3 + 2] = s6;
      }
      if (a.tp_world && a.tp_stats[0]) {
        const int num = tp_number(a);
        for (int r = 0; r < a.tp_world; ++r) {
          tp_store(a.tp_stats[r] + tile * 3 + 0, tp_pair(s2, num));
          tp_store(a.tp_stats[r] + tile * 3 + 1, tp_pair(s4, num));
          tp_store(a.tp_stats[r] + tile * 3 + 2, tp_pair(s6, num));
        }
      }
    }
  }
  if ((a.argmax_out || a.argmax_key_out) && any) {
    // Key of this lane's row: value bits mapped to an unsigned order (NaN as -inf) above the
    // inverted row index, so the largest key is the largest value at its first index.
    unsigned long long key = 0;
    if (have && row < a.N) {
      float f = __half2float(hv);
      if (isnan(f)) f = -INFINITY;
      const uint32_t b = __float_as_uint(f);
      const uint32_t hi = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
      key = ((unsigned long long)hi << 32) | (0xFFFFFFFFu - (uint32_t)(row + a.argmax_row_offset));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
    if (lane == 0) {
      atomicMax(a.amax_key, key);
      __threadfence();
      if (atomicAdd(a.amax_tiles, 1) == a.ntiles - 1) {
        // every tile's key is in: publish the token and reset the state
        __threadfence();
        const unsigned long long k = atomicExch(a.amax_key, 0ull);
        atomicExch(a.amax_tiles, 0);
        if (a.argmax_key_out) *a.argmax_key_out = (long long)(k ^ 0x8000000000000000ull);
        if (a.argmax_out) a.argmax_out[0] = k == 0 ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        if (a.pos_len_inc) {
          a.pos_len_inc[0] += 1;
          a.pos_len_inc[1] += 1;
        }
      }
    }
  }
}

// Build x (full K) in shared memory: each 8-value word permuted to the nibble order
// the dequant produces (0,4,1,5,2,6,3,7), plus per-group sums of x.
// V2 (TMA kernel) also pre-scales the odd-k ("hi" nibble) values by 1/16 and
// writes corr[g] = 1024·Σ(stored values of group g): the dequant there feeds the
// MMA 1024+q (even k) and 1024+16q (odd k), so Σ q·x = C − corr exactly.
//
// One round trip to memory: every input word a thread needs (at most
// kMaxStageWords, i.e. K ≤ 8·256·kMaxStageWords) is loaded into registers
// first; the row statistics are reduced from those registers; group sums come
// from shuffles over the 8 consecutive threads that hold one group's words.
// Largest K (in 8-value words per thread of a 256-thread CTA) each prologue supports.
template <int MODE>
struct StageWords {
  static constexpr int value = MODE == 1 ? 4 : 8;
};

// `after_issue` runs on every thread once the input loads are in flight (the TMA
// kernel issues the rest of its weight prefetch there, behind the staging loads).
// A prologue's constant inputs — the RMSNorm weight words a thread stages (mode 1) and the
// PolyNorm weights and bias (mode 2) — read before the kernel waits for the previous one: they
// are model weights that no kernel of the step writes, and reading them after the wait put a
// DRAM miss on the staging's critical path.
template <int MODE>
struct StageConst {
  uint4 norm[StageWords<MODE>::value];
  float poly[4];
};

template <int MODE>
__device__ __forceinline__ void stage_const_load(const LinArgs& a, StageConst<MODE>& c) {
  if constexpr (MODE == kModeAddRms) {
    const int words = (int)(a.K / 8);
#pragma unroll
    for (int i = 0; i < StageWords<MODE>::value; ++i) {
      const int wi = threadIdx.x + i * blockDim.x;
      if (wi < words) c.norm[i] = *reinterpret_cast<const uint4*>(a.norm_w + (int64_t)wi * 8);
    }
  } else if constexpr (MODE == kModePoly) {
    c.poly[0] = __half2float(a.poly_w[0]);
    c.poly[1] = __half2float(a.poly_w[1]);
    c.poly[2] = __half2float(a.poly_w[2]);
    c.poly[3] = __half2float(a.poly_b[0]);
  }
}

template <int MODE, bool V2, typename AfterIssue>
__device__ void stage_x(const LinArgs& a, __half* xp_s, float* xsum_s, float* corr_s, float* red, __half* delta_s,
                        AfterIssue&& after_issue, const StageConst<MODE>* pre = nullptr) {
  constexpr int kMaxStageWords = StageWords<MODE>::value;
  const int64_t K = a.K;
  const int words = (int)(K / 8);
  const int nthr = blockDim.x;
  const int tid = threadIdx.x;
  const __half* delta = a.delta;
  if (MODE == kModeAddRms && a.tp_in) {
    // Tensor-parallel consumer: delta = fp16(Σ_r partial_r) over the ranks' exchanged rows,
    // summed in rank order so every rank gets the same bits.
    const unsigned long long t_read = global_ns();
    const int num = tp_number(a);
    for (int w = tid; w < words; w += nthr) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int r = 0; r < a.tp_world; ++r) {
        // 8 pairs = four 16-byte loads of two 64-bit pairs each; a pair not yet carrying this
        // number is re-read alone
        const long long* p = a.tp_in + (int64_t)r * K + (int64_t)w * 8;
        long long q[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) tp_load2(p + 2 * j, q[2 * j], q[2 * j + 1]);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          acc[j] += (int)(q[j] >> 32) == num ? __uint_as_float((uint32_t)q[j]) : tp_read(p + j, num, a.err);
      }
      store_vec<__half, 8>(delta_s + (int64_t)w * 8, acc);
    }
    __syncthreads();
    if (blockIdx.x == 0 && tid == 0 && a.tp_wait_ns) atomicAdd(a.tp_wait_ns, global_ns() - t_read);
    delta = delta_s;
  }
  uint4 in0[kMaxStageWords], in1[kMaxStageWords], in2[kMaxStageWords];
  const __half* hsrc = a.h_in;
  float stats_acc[3] = {0.f, 0.f, 0.f};
  if (MODE == kModeAddRms && a.token) {
    int64_t t = a.token[0];
    if (t < 0 || t >= a.vocab) t = 0;  // out-of-range ids read row 0
    hsrc = a.embed + t * K;
  }
  // ---- issue every load ----
#pragma unroll
  for (int i = 0; i < kMaxStageWords; ++i) {
    const int wi = tid + i * nthr;
    if (wi < words) {
      if constexpr (MODE == kModeX) {
        in0[i] = *reinterpret_cast<const uint4*>(a.x + (int64_t)wi * 8);
      } else if constexpr (MODE == kModeAddRms) {
        in0[i] = *reinterpret_cast<const uint4*>(hsrc + (int64_t)wi * 8);
        in1[i] = delta ? *reinterpret_cast<const uint4*>(delta + (int64_t)wi * 8) : make_uint4(0, 0, 0, 0);
        in2[i] = pre ? pre->norm[i] : *reinterpret_cast<const uint4*>(a.norm_w + (int64_t)wi * 8);
      } else {
        in0[i] = *reinterpret_cast<const uint4*>(a.gate + (int64_t)wi * 8);
        in1[i] = *reinterpret_cast<const uint4*>(a.up + (int64_t)wi * 8);
      }
    }
  }
  if (MODE == kModePoly) {
    if (a.tp_stats_in) {  // all ranks' tile statistics, exchanged as pairs
      const unsigned long long t_read = global_ns();
      const int num = tp_number(a);
      for (int i = tid; i < a.stats_count; i += nthr) {
        stats_acc[0] += tp_read(a.tp_stats_in + i * 3 + 0, num, a.err);
        stats_acc[1] += tp_read(a.tp_stats_in + i * 3 + 1, num, a.err);
        stats_acc[2] += tp_read(a.tp_stats_in + i * 3 + 2, num, a.err);
      }
      if (blockIdx.x == 0 && tid == 0 && a.tp_wait_ns) atomicAdd(a.tp_wait_ns, global_ns() - t_read);
    } else {
      // The first rounds' loads all go out before any is summed (one L2 round trip instead of
      // one per round); the summation order is the plain loop's.
      constexpr int kRounds = 4;
      float sv[kRounds][3];
#pragma unroll
      for (int j = 0; j < kRounds; ++j) {
        const int i = tid + j * nthr;
        if (i < a.stats_count) {
          sv[j][0] = a.stats[i * 3 + 0];
          sv[j][1] = a.stats[i * 3 + 1];
          sv[j][2] = a.stats[i * 3 + 2];
        }
      }
#pragma unroll
      for (int j = 0; j < kRounds; ++j) {
        if (tid + j * nthr < a.stats_count) {
          stats_acc[0] += sv[j][0];
          stats_acc[1] += sv[j][1];
          stats_acc[2] += sv[j][2];
        }
      }
      for (int i = tid + kRounds * nthr; i < a.stats_count; i += nthr) {
        stats_acc[0] += a.stats[i * 3 + 0];
        stats_acc[1] += a.stats[i * 3 + 1];
        stats_acc[2] += a.stats[i * 3 + 2];
      }
    }
  }
  after_issue();
  // ---- row statistics ----
  float inv = 1.f, r2 = 0.f, r4 = 0.f, r6 = 0.f, pw0 = 0.f, pw1 = 0.f, pw2 = 0.f, pb = 0.f;
  if (MODE == kModeAddRms) {
    float acc[1] = {0.f};
#pragma unroll
    for (int i = 0; i < kMaxStageWords; ++i) {
      if (tid + i * nthr < words) {
        const __half2* hv = reinterpret_cast<const __half2*>(&in0[i]);
        const __half2* dv = reinterpret_cast<const __half2*>(&in1[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 v = __half22float2(delta ? __hadd2(hv[j], dv[j]) : hv[j]);
          acc[0] += v.x * v.x;
          acc[0] += v.y * v.y;
        }
      }
    }
    block_sum<1>(acc, red);
    inv = rsqrtf(acc[0] / (float)K + a.eps);
  } else if (MODE == kModePoly) {
    block_sum<3>(stats_acc, red);
    r2 = rsqrtf(stats_acc[0] * a.poly_inv_dim + a.poly_eps);
    r4 = rsqrtf(stats_acc[1] * a.poly_inv_dim + a.poly_eps);
    r6 = rsqrtf(stats_acc[2] * a.poly_inv_dim + a.poly_eps);
    pw0 = pre ? pre->poly[0] : __half2float(a.poly_w[0]);
    pw1 = pre ? pre->poly[1] : __half2float(a.poly_w[1]);
    pw2 = pre ? pre->poly[2] : __half2float(a.poly_w[2]);
    pb = pre ? pre->poly[3] : __half2float(a.poly_b[0]);
  }
  const bool write_h = MODE == kModeAddRms && a.h_out && blockIdx.x == 0;
  // ---- build x, permute, group sums ----
  // In half2 pairs: the fp16 residual add (__hadd2) and PolyNorm·up product (__hmul2) equal
  // rounding the fp32 sum/product once (fp32 holds the exact product of two fp16 values, and
  // its 24 bits make the fp32-then-fp16 rounding of a sum innocuous), and pairs of floats are
  // rounded to fp16 with one packed conversion.
#pragma unroll
  for (int i = 0; i < kMaxStageWords; ++i) {
    const int wi = tid + i * nthr;
    if (i * nthr >= words) break;  // uniform across the block
    const bool act = wi < words;
    __half2 h2[4];
    if (act) {
      const __half2* e0 = reinterpret_cast<const __half2*>(&in0[i]);
      const __half2* e1 = reinterpret_cast<const __half2*>(&in1[i]);
      const __half2* e2 = reinterpret_cast<const __half2*>(&in2[i]);
      if constexpr (MODE == kModeX) {
#pragma unroll
        for (int j = 0; j < 4; ++j) h2[j] = e0[j];
      } else if constexpr (MODE == kModeAddRms) {
        __half2 vh[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) vh[j] = delta ? __hadd2(e0[j], e1[j]) : e0[j];
        if (write_h) *reinterpret_cast<uint4*>(a.h_out + (int64_t)wi * 8) = *reinterpret_cast<const uint4*>(vh);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 v = __half22float2(vh[j]);
          const float2 w = __half22float2(e2[j]);
          h2[j] = __floats2half2_rn(v.x * inv * w.x, v.y * inv * w.y);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 g = __half22float2(e0[j]);
          const float gx2 = g.x * g.x, gy2 = g.y * g.y;
          const float gx3 = gx2 * g.x, gy3 = gy2 * g.y;
          const float px = pw0 * (gx3 * r6) + pw1 * (gx2 * r4) + pw2 * (g.x * r2) + pb;
          const float py = pw0 * (gy3 * r6) + pw1 * (gy2 * r4) + pw2 * (g.y * r2) + pb;
          h2[j] = __hmul2(__floats2half2_rn(px, py), e1[j]);
        }
      }
      if (V2) {  // odd k (the .y halves) pre-scaled by 1/16, an exact power of two
        const __half2 scale = __halves2half2(__float2half_rn(1.f), __float2half_rn(0.0625f));
#pragma unroll
        for (int j = 0; j < 4; ++j) h2[j] = __hmul2(h2[j], scale);
      }
      // dequant order of the 8 values: 0,4,1,5,2,6,3,7
      uint4 o;
      __half2* oe = reinterpret_cast<__half2*>(&o);
      oe[0] = __lows2half2(h2[0], h2[2]);
      oe[1] = __highs2half2(h2[0], h2[2]);
      oe[2] = __lows2half2(h2[1], h2[3]);
      oe[3] = __highs2half2(h2[1], h2[3]);
      *reinterpret_cast<uint4*>(xp_s + (int64_t)wi * 8 + (V2 ? (int64_t)(wi >> 3) * (kXGroupBytes / 2 - 64) : 0)) = o;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) h2[j] = __float2half2_rn(0.f);
    }
    // even-k (lo) and odd-k (hi) sums of this word, reduced over the group's 8 threads
    float lo = 0.f, hi = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h2[j]);
      lo += f.x;
      hi += f.y;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      lo += __shfl_xor_sync(0xffffffffu, lo, o);
      hi += __shfl_xor_sync(0xffffffffu, hi, o);
    }
    if (act && (wi & 7) == 0) {
      const int g = wi >> 3;
      if (V2) {
        xsum_s[g] = lo + 16.f * hi;
        corr_s[g] = 1024.f * (lo + hi);
      } else {
        xsum_s[g] = lo + hi;
      }
    }
  }
  __syncthreads();
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 2) q4_gemv_kernel(LinArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* xp_s = reinterpret_cast<__half*>(smem_raw);
  float* xsum_s = reinterpret_cast<float*>(smem_raw + (size_t)a.K * sizeof(__half));
  float* red = xsum_s + a.K / 64;
  __half* delta_s = reinterpret_cast<__half*>(red + 32 * 3);  // K halves when a.tp_in is set

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int gw = blockIdx.x * kWarps + warp;
  const uint32_t units = (uint32_t)a.units, tw = (uint32_t)a.total_warps;
  const int u0 = gw < a.total_warps ? (int)((uint32_t)gw * units / tw) : (int)units;
  const int u1 = gw < a.total_warps ? (int)((uint32_t)(gw + 1) * units / tw) : (int)units;
  const int nblk = a.nblk;
  const int diff = r - (c >> 1);
  const int q_lane = (diff >= 0 && (diff & 1) == 0) ? diff >> 1 : -1;

  // Weights do not depend on the previous kernel: start streaming them first.
  UnitRegs A, B;
  int tile = u0 / nblk, blk = u0 - (u0 / nblk) * nblk;
  if (u0 < u1) load_unit(A, a, tile, blk, r, c);
  grid_dep_wait();
  grid_dep_launch();
  stage_x<MODE, false>(a, xp_s, xsum_s, nullptr, red, delta_s, [] {});

  float acc_r = 0.f, acc_r8 = 0.f;
  for (int u = u0; u < u1; u += 2) {
    const bool has1 = u + 1 < u1;
    int t1 = tile, b1 = blk + 1;
    if (b1 == nblk) { b1 = 0; ++t1; }
    if (has1) load_unit(B, a, t1, b1, r, c);
    compute_unit(A, a, blk, xp_s, xsum_s, c, q_lane, acc_r, acc_r8);
    if (!has1 || t1 != tile) {
      tile_epilogue<2>(a, tile, gw, acc_r, acc_r8, lane);
      acc_r = acc_r8 = 0.f;
    }
    if (has1) {
      int t2 = t1, b2 = b1 + 1;
      if (b2 == nblk) { b2 = 0; ++t2; }
      if (u + 2 < u1) load_unit(A, a, t2, b2, r, c);
      compute_unit(B, a, b1, xp_s, xsum_s, c, q_lane, acc_r, acc_r8);
      if (u + 2 >= u1 || t2 != t1) {
        tile_epilogue<2>(a, t1, gw, acc_r, acc_r8, lane);
        acc_r = acc_r8 = 0.f;
      }
      tile = t2;
      blk = b2;
    }
  }
}

// ---- TMA variant: weights arrive in shared memory through a per-warp ring ------
//
// 8 warps per CTA and one CTA per SM, with a footprint (≈110 KB shared, 128
// registers) that leaves room for the next kernel's CTA: launched with
// programmatic serialization, it starts its own weight prefetch while this one
// finishes. Each warp owns kStages ring slots of one
// unit each — codes as two 128B-swizzled boxes of 16 rows × 128 B (so the
// lanes' 8-byte reads are spread over the banks), scales and biases as
// 16 × 16 B boxes — filled by 2D tiled TMA loads straight from the MLX layout
// and tracked by one mbarrier per slot. Lane 0 refills a slot with the unit
// kStages ahead as soon as the warp has read it.
//
// Compute: one MMA quad per quantization group. Lane (r, c) takes the 16
// consecutive k of group g at 16c (two words per row), so a step's 16 k all
// belong to one group and every B column carries the full x: C's columns are
// all the group's dot products. Nibbles enter the MMA as fp16 1024+q (even k)
// or 1024+16q (odd k, against x/16) — one LOP3 per nibble pair — and the
// per-group constant 1024·Σx' is subtracted after the quad. Eight independent
// quads per unit keep the tensor pipe and the scheduler busy.
//
// All mbarrier waits are bounded: on time-out the kernel records an error in
// the workspace, lets its in-flight copies land (bounded) and stops.
#ifndef MOTIF_GEMV_TMA_WARPS
#define MOTIF_GEMV_TMA_WARPS 16
#endif
#ifndef MOTIF_GEMV_STAGES
#define MOTIF_GEMV_STAGES 2
#endif
constexpr int kTmaWarps = MOTIF_GEMV_TMA_WARPS;
constexpr int kTmaThreads = kTmaWarps * 32;
constexpr int kStages = MOTIF_GEMV_STAGES;
// Two CTAs per SM (so the next GEMV's prefetch can co-reside) when the ring is small enough.
constexpr int kTmaMinBlocks = kTmaWarps * kStages <= 16 ? 2 : 1;
constexpr int kTmaSmemCap = kTmaMinBlocks == 2 ? 113 * 1024 : 225 * 1024;
constexpr int kSlotBytes = 5120;  // 2 × 2048 codes + 256 scales + 256 biases, 1 KiB aligned
constexpr int kMaxPolls = 1 << 20;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < kMaxPolls; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.b32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// A 2D tiled TMA load with an L2 eviction-priority policy (createpolicy): the weight stream is read once
// per step, so its lines are marked first to be evicted and the small vectors the kernels read
// and write between launches (activations, norm weights, statistics, counters) stay in L2.
__device__ __forceinline__ void tma_load_2d_stream(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                                   uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}

__device__ __forceinline__ void issue_unit(const LinArgs& a, int tile, int blk, uint32_t slot, uint32_t bar) {
  const uint64_t pol = evict_first_policy();
  mbar_expect_tx(bar, 4096 + 256 + 256);
  tma_load_2d_stream(slot, &a.tm_w, blk * 256, tile * kTileRows, bar, pol);
  tma_load_2d_stream(slot + 2048, &a.tm_w, blk * 256 + 128, tile * kTileRows, bar, pol);
  tma_load_2d_stream(slot + 4096, &a.tm_s, blk * 16, tile * kTileRows, bar, pol);
  tma_load_2d_stream(slot + 4352, &a.tm_b, blk * 16, tile * kTileRows, bar, pol);
}

__device__ __forceinline__ uint2 lds64(const unsigned char* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Word of 8 nibbles -> (1024+n0, 1024+n4) (1024+16n1, 1024+16n5) (1024+n2, 1024+n6) (1024+16n3, 1024+16n7).
__device__ __forceinline__ void dequant_word_offset(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t LO = 0x000F000Fu, HI = 0x00F000F0u, EX = 0x64006400u;
  p[0] = lop3_and_or(w, LO, EX);
  p[1] = lop3_and_or(w, HI, EX);
  const uint32_t w8 = w >> 8;
  p[2] = lop3_and_or(w8, LO, EX);
  p[3] = lop3_and_or(w8, HI, EX);
}

// One unit (16 rows × 8 groups of 64) on the tensor pipe, one B column per group.
//
// Lane (r, c) supplies the A operand for rows r and r+8 of group c (MMAs into Ca)
// and group c+4 (MMAs into Cb): the 32 code bytes of each, chunks 2c and 2c+1 of
// the 128B-swizzled box. B column n is fed by the lanes with r == n; only the
// quad-diagonal lane (r == c) holds x (the group's staged values, `xl`), every
// other lane reads zeros, so column n of Ca/Cb accumulates exactly the dot of
// group n / n+4 and the accumulators stay live for the whole unit. Lanes c < 2
// then hold groups 2c, 2c+1 (Ca) and 2c+4, 2c+5 (Cb) of rows r and r+8 and apply
// the affine epilogue s·(C − corr) + b·Σx once per unit.
__device__ __forceinline__ void compute_unit_tma(const unsigned char* slot, const unsigned char* xl, uint32_t o0,
                                                 uint32_t o1, int r, int c, int blk,
                                                 const float* __restrict__ xsum_s, const float* __restrict__ corr_s,
                                                 float& acc_r, float& acc_r8) {
  float Ca[4] = {0.f, 0.f, 0.f, 0.f}, Cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int h = 0; h < 2; ++h) {  // words 4h .. 4h+3 of each group
    const uint32_t o = h ? o1 : o0;
    const uint4 wa = lds128(slot + o), wa8 = lds128(slot + 1024 + o);
    const uint4 wb = lds128(slot + 2048 + o), wb8 = lds128(slot + 3072 + o);
    uint4 xa[4], xb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xa[i] = lds128(xl + h * 64 + i * 16);
      xb[i] = lds128(xl + 4 * kXGroupBytes + h * 64 + i * 16);
    }
    const uint32_t* pa = &wa.x;
    const uint32_t* pa8 = &wa8.x;
    const uint32_t* pb = &wb.x;
    const uint32_t* pb8 = &wb8.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t P[4], P8[4], Q[4], Q8[4];
      dequant_word_offset(pa[i], P);
      dequant_word_offset(pa8[i], P8);
      dequant_word_offset(pb[i], Q);
      dequant_word_offset(pb8[i], Q8);
      mma16816(Ca, P[0], P8[0], P[1], P8[1], xa[i].x, xa[i].y);
      mma16816(Cb, Q[0], Q8[0], Q[1], Q8[1], xb[i].x, xb[i].y);
      mma16816(Ca, P[2], P8[2], P[3], P8[3], xa[i].z, xa[i].w);
      mma16816(Cb, Q[2], Q8[2], Q[3], Q8[3], xb[i].z, xb[i].w);
    }
  }
  if (c < 2) {
    const int g = blk * 8 + 2 * c;
    const float2 cra = *reinterpret_cast<const float2*>(corr_s + g);
    const float2 crb = *reinterpret_cast<const float2*>(corr_s + g + 4);
    const float2 xsa = *reinterpret_cast<const float2*>(xsum_s + g);
    const float2 xsb = *reinterpret_cast<const float2*>(xsum_s + g + 4);
    const unsigned char* sp = slot + 4096 + r * 16 + 4 * c;  // scales of row r, groups 2c and 2c+1
    const float2 sa = __half22float2(*reinterpret_cast<const __half2*>(sp));
    const float2 sb = __half22float2(*reinterpret_cast<const __half2*>(sp + 8));
    const float2 sa8 = __half22float2(*reinterpret_cast<const __half2*>(sp + 128));
    const float2 sb8 = __half22float2(*reinterpret_cast<const __half2*>(sp + 136));
    const float2 ba = __half22float2(*reinterpret_cast<const __half2*>(sp + 256));
    const float2 bb = __half22float2(*reinterpret_cast<const __half2*>(sp + 264));
    const float2 ba8 = __half22float2(*reinterpret_cast<const __half2*>(sp + 384));
    const float2 bb8 = __half22float2(*reinterpret_cast<const __half2*>(sp + 392));
    acc_r += sa.x * (Ca[0] - cra.x) + ba.x * xsa.x + sa.y * (Ca[1] - cra.y) + ba.y * xsa.y +
             sb.x * (Cb[0] - crb.x) + bb.x * xsb.x + sb.y * (Cb[1] - crb.y) + bb.y * xsb.y;
    acc_r8 += sa8.x * (Ca[2] - cra.x) + ba8.x * xsa.x + sa8.y * (Ca[3] - cra.y) + ba8.y * xsa.y +
              sb8.x * (Cb[2] - crb.x) + bb8.x * xsb.x + sb8.y * (Cb[3] - crb.y) + bb8.y * xsb.y;
  }
}

template <int MODE>
__global__ void __launch_bounds__(kTmaThreads, kTmaMinBlocks) q4_gemv_tma_kernel(const __grid_constant__ LinArgs a) {
  // 1 KiB alignment (128B-swizzled TMA boxes); plain pointer arithmetic on the shared
  // array keeps every slot/x access a shared-memory load.
  extern __shared__ __align__(1024) unsigned char smem_tma[];
  unsigned char* ring = smem_tma;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + (size_t)kTmaWarps * kStages * kSlotBytes);
  __half* xp_s = reinterpret_cast<__half*>(bars + kTmaWarps * kStages);
  // zero_s is offset 64 B (mod 128) from the x rows so its broadcast read never shares a
  // bank with the diagonal lanes' x reads.
  unsigned char* zero_s = reinterpret_cast<unsigned char*>(xp_s) + (size_t)(a.K / 64) * kXGroupBytes + 64;
  float* xsum_s = reinterpret_cast<float*>(zero_s + kZeroBytes);
  float* corr_s = xsum_s + a.K / 64;
  float* red = corr_s + a.K / 64;
  __half* delta_s = reinterpret_cast<__half*>(red + 32 * 3);  // K halves when a.tp_in is set

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int gw = blockIdx.x * kTmaWarps + warp;
  const uint32_t units = (uint32_t)a.units, tw = (uint32_t)a.total_warps;
  const int u0 = gw < a.total_warps ? (int)((uint32_t)gw * units / tw) : (int)units;
  const int u1 = gw < a.total_warps ? (int)((uint32_t)(gw + 1) * units / tw) : (int)units;
  const int nblk = a.nblk;
  unsigned char* my_ring = ring + (size_t)warp * kStages * kSlotBytes;
  uint64_t* my_bars = bars + warp * kStages;

  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&a.tm_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&a.tm_s)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&a.tm_b)) : "memory");
  }
  if (lane == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(smem_u32(&my_bars[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncwarp();
  // (tile, blk) of the next unit to fetch. Weights do not depend on the previous
  // kernel: the first slot is filled before waiting for it, the others right after
  // the x inputs are requested, so the staging loads queue behind one unit per warp
  // instead of the whole ring. A plain-x linear (mode 0: the o projection after the
  // attention step) fills the whole ring before waiting: its staging is one L2-resident
  // vector, and its CTAs start on the SMs the attention step leaves free, so most of
  // its weights arrive while the attention still runs.
  constexpr int kPreSlots = MODE == kModeX ? kStages : 1;
  int it = u0 / nblk, ib = u0 - (u0 / nblk) * nblk;
  if (lane == 0) {
    for (int i = 0; i < kPreSlots && u0 + i < u1; ++i) {
      issue_unit(a, it, ib, smem_u32(my_ring + i * kSlotBytes), smem_u32(&my_bars[i]));
      if (++ib == nblk) { ib = 0; ++it; }
    }
  }
  StageConst<MODE> cst;
  stage_const_load<MODE>(a, cst);
  for (int i = threadIdx.x; i < kZeroBytes / 16; i += blockDim.x) reinterpret_cast<uint4*>(zero_s)[i] = make_uint4(0, 0, 0, 0);
  grid_dep_wait();
  grid_dep_launch();
  stage_x<MODE, true>(a, xp_s, xsum_s, corr_s, red, delta_s, [&] {
    if (lane == 0) {
      for (int i = kPreSlots; i < kStages && u0 + i < u1; ++i) {
        issue_unit(a, it, ib, smem_u32(my_ring + i * kSlotBytes), smem_u32(&my_bars[i]));
        if (++ib == nblk) { ib = 0; ++it; }
      }
    }
  }, &cst);
  // Per-lane operand addresses (see compute_unit_tma).
  const uint32_t o0 = r * 128 + (((2 * c) ^ r) * 16), o1 = r * 128 + (((2 * c + 1) ^ r) * 16);
  const bool diag = r == c;
  const unsigned char* xrow = reinterpret_cast<const unsigned char*>(xp_s) + c * kXGroupBytes;

  float acc_r = 0.f, acc_r8 = 0.f;
  bool ok = true;
  int tile = u0 / nblk, blk = u0 - (u0 / nblk) * nblk;
  for (int u = u0; u < u1; ++u) {
    const int j = u - u0;
    const int slot = j % kStages;
    if (!mbar_wait(smem_u32(&my_bars[slot]), (uint32_t)((j / kStages) & 1))) {
      ok = false;
      // Let the copies still in flight (units after u, at most kStages-1) land before exiting (bounded).
      for (int v = u + 1; v < u1 && v < u + kStages; ++v) {
        const int jv = v - u0;
        mbar_wait(smem_u32(&my_bars[jv % kStages]), (uint32_t)((jv / kStages) & 1));
      }
      break;
    }
    const unsigned char* xl = diag ? xrow + blk * 8 * kXGroupBytes : zero_s;
    compute_unit_tma(my_ring + slot * kSlotBytes, xl, o0, o1, r, c, blk, xsum_s, corr_s, acc_r, acc_r8);
    __syncwarp();
    if (lane == 0 && u + kStages < u1) {
      issue_unit(a, it, ib, smem_u32(my_ring + slot * kSlotBytes), smem_u32(&my_bars[slot]));
      if (++ib == nblk) { ib = 0; ++it; }
    }
    if (u + 1 >= u1 || blk + 1 == nblk) {
      tile_epilogue<16>(a, tile, gw, acc_r, acc_r8, lane);
      acc_r = acc_r8 = 0.f;
    }
    if (++blk == nblk) { blk = 0; ++tile; }
  }
  if (!ok && lane == 0 && a.err) atomicExch(a.err, 1);
}

// ---- several x rows at once: the [1, K+1] speculative verify, short prompt blocks ------------
//
// The weight stream of q4_gemv_tma_kernel (units of 16 rows × 512 k, a per-warp TMA ring,
// stream-K over the grid), but the MMA's eight B columns are up to eight x rows instead of the
// eight groups of a unit. Lane (r, c) feeds rows r and r+8 with words 2c and 2c+1 of ONE group
// per quad of MMAs, so each MMA's 16 k values all belong to that group and C[row][x row] is
// the group's exact dot; the MLX affine epilogue s·(C − corr) + b·Σx then runs per group and
// per x row. Every weight byte is streamed once for all the rows. x rows are staged like the
// one-row kernel's x (dequant order 0,4,1,5,.., odd k pre-scaled by 1/16), one row every 2K + 16
// bytes so the eight rows spread over the banks; per group, the float4 {corr, Σx} of x rows 2c
// and 2c+1 (corr = 1024·Σ of the staged values, the dequant offset) sits where lane c reads it
// with one load, and the MMA accumulator starts at −corr so only s·C + b·Σx remains per group.
constexpr int kRowsMax = 8;
constexpr int kRowsSmemCap = 225 * 1024;  // one CTA per SM

// Ring slots, then their barriers rounded up to 128 B, then the staged rows.
__host__ __device__ inline size_t rows_xs_offset(int warps) {
  return (size_t)warps * kStages * kSlotBytes + (((size_t)warps * kStages * 8 + 127) & ~(size_t)127);
}

size_t rows_xbytes(int64_t K, int R) { return (size_t)R * ((size_t)K * 2 + 16) + (size_t)(K / 64) * 64; }

size_t rows_smem_bytes(int64_t K, int R, int warps) { return rows_xs_offset(warps) + rows_xbytes(K, R); }

// Warps per CTA (up to 16) that fit beside the staged rows (each takes kStages ring slots).
int rows_warps(int64_t K, int R) {
  int w = 16;
  while (w > 0 && rows_smem_bytes(K, R, w) > (size_t)kRowsSmemCap) --w;
  return w;
}

// fp16 half `hi` (0 = low 16 bits) of a packed pair, as float.
__device__ __forceinline__ float half_of(uint32_t w, int hi) {
  return __half2float(__ushort_as_half((unsigned short)(hi ? w >> 16 : w & 0xFFFFu)));
}

template <int R>
__global__ void __launch_bounds__(512, 1) q4_gemv_rows_kernel(const __grid_constant__ LinArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_rows[];
  const int nw = blockDim.x >> 5;
  unsigned char* ring = smem_rows;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + (size_t)nw * kStages * kSlotBytes);
  unsigned char* xs = smem_rows + rows_xs_offset(nw);
  const int64_t K = a.K;
  const int G = (int)(K / 64);
  const int64_t xstride = K * 2 + 16;
  float4* cx_s = reinterpret_cast<float4*>(xs + R * xstride);  // [G][4]: {corr, Σx} of x rows 2c, 2c+1

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int gw = blockIdx.x * nw + warp;
  const uint32_t units = (uint32_t)a.units, tw = (uint32_t)a.total_warps;
  const int u0 = gw < a.total_warps ? (int)((uint32_t)gw * units / tw) : (int)units;
  const int u1 = gw < a.total_warps ? (int)((uint32_t)(gw + 1) * units / tw) : (int)units;
  const int nblk = a.nblk;
  unsigned char* my_ring = ring + (size_t)warp * kStages * kSlotBytes;
  uint64_t* my_bars = bars + warp * kStages;

  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&a.tm_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&a.tm_s)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&a.tm_b)) : "memory");
  }
  if (lane == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(smem_u32(&my_bars[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncwarp();
  // weights do not depend on the previous kernel: fill the ring before waiting for it
  int it = u0 / nblk, ib = u0 - (u0 / nblk) * nblk;
  if (lane == 0) {
    for (int i = 0; i < kStages && u0 + i < u1; ++i) {
      issue_unit(a, it, ib, smem_u32(my_ring + i * kSlotBytes), smem_u32(&my_bars[i]));
      if (++ib == nblk) { ib = 0; ++it; }
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  // ---- stage the x rows: one (group, row pair) per thread step ----
  const __half sixteenth = __float2half_rn(0.0625f);
  for (int i = threadIdx.x; i < 4 * G; i += blockDim.x) {
    const int g = i >> 2, pair = i & 3;
    float cx[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int row = 2 * pair + h2;
      if (row >= R) break;
      const __half* src = a.x + (int64_t)row * K + (int64_t)g * 64;
      unsigned char* dst = xs + row * xstride + (int64_t)g * 128;
      float lo = 0.f, hi = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const uint4 v = *reinterpret_cast<const uint4*>(src + w * 8);
        const __half* e = reinterpret_cast<const __half*>(&v);
        __half h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = (j & 1) ? __hmul(e[j], sixteenth) : e[j];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          lo += __half2float(h[j]);
          hi += __half2float(h[j + 1]);
        }
        uint4 o;
        __half* oe = reinterpret_cast<__half*>(&o);
        oe[0] = h[0]; oe[1] = h[4]; oe[2] = h[1]; oe[3] = h[5];
        oe[4] = h[2]; oe[5] = h[6]; oe[6] = h[3]; oe[7] = h[7];
        *reinterpret_cast<uint4*>(dst + w * 16) = o;
      }
      cx[2 * h2] = 1024.f * (lo + hi);
      cx[2 * h2 + 1] = lo + 16.f * hi;
    }
    cx_s[i] = make_float4(cx[0], cx[1], cx[2], cx[3]);
  }
  __syncthreads();

  const int n0 = 2 * c, n1 = 2 * c + 1;  // this lane's x rows in C
  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // (row r, n0) (row r, n1) (row r+8, n0) (row r+8, n1)
  bool ok = true;
  int tile = u0 / nblk, blk = u0 - (u0 / nblk) * nblk;
  for (int u = u0; u < u1; ++u) {
    const int j = u - u0;
    const int slot_i = j % kStages;
    if (!mbar_wait(smem_u32(&my_bars[slot_i]), (uint32_t)((j / kStages) & 1))) {
      ok = false;
      for (int v = u + 1; v < u1 && v < u + kStages; ++v) {
        const int jv = v - u0;
        mbar_wait(smem_u32(&my_bars[jv % kStages]), (uint32_t)((jv / kStages) & 1));
      }
      break;
    }
    const unsigned char* slot = my_ring + slot_i * kSlotBytes;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {  // groups 4·half .. 4·half+3 (one 128B-swizzled box)
      // fp16 scales / biases of rows r and r+8 for these four groups
      const unsigned char* sp = slot + 4096 + r * 16 + half * 8;
      const uint2 sr = lds64(sp), sr8 = lds64(sp + 128), br = lds64(sp + 256), br8 = lds64(sp + 384);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int gi = 4 * half + q;
        const int chunk = 2 * q + (c >> 1);
        const uint32_t off = (gi >> 2) * 2048 + r * 128 + ((chunk ^ r) << 4) + (c & 1) * 8;
        const uint2 wr = lds64(slot + off), wr8 = lds64(slot + off + 1024);
        uint32_t P0[4], P1[4], Q0[4], Q1[4];
        dequant_word_offset(wr.x, P0);
        dequant_word_offset(wr.y, P1);
        dequant_word_offset(wr8.x, Q0);
        dequant_word_offset(wr8.y, Q1);
        const int gg = blk * 8 + gi;
        uint4 b0 = make_uint4(0, 0, 0, 0), b1 = make_uint4(0, 0, 0, 0);
        if (r < R) {
          const unsigned char* xp = xs + r * xstride + (int64_t)gg * 128 + c * 32;
          b0 = lds128(xp);
          b1 = lds128(xp + 16);
        }
        const float4 cx = cx_s[gg * 4 + c];  // {corr, Σx} of x rows n0, n1 (zeros past R)
        float C[4] = {-cx.x, -cx.z, -cx.x, -cx.z};
        mma16816(C, P0[0], Q0[0], P0[1], Q0[1], b0.x, b0.y);
        mma16816(C, P0[2], Q0[2], P0[3], Q0[3], b0.z, b0.w);
        mma16816(C, P1[0], Q1[0], P1[1], Q1[1], b1.x, b1.y);
        mma16816(C, P1[2], Q1[2], P1[3], Q1[3], b1.z, b1.w);
        const uint32_t ws = (q & 2) ? sr.y : sr.x, ws8 = (q & 2) ? sr8.y : sr8.x;
        const uint32_t wb = (q & 2) ? br.y : br.x, wb8 = (q & 2) ? br8.y : br8.x;
        const float s_r = half_of(ws, q & 1), s_r8 = half_of(ws8, q & 1);
        const float b_r = half_of(wb, q & 1), b_r8 = half_of(wb8, q & 1);
        acc[0] = fmaf(s_r, C[0], fmaf(b_r, cx.y, acc[0]));
        acc[1] = fmaf(s_r, C[1], fmaf(b_r, cx.w, acc[1]));
        acc[2] = fmaf(s_r8, C[2], fmaf(b_r8, cx.y, acc[2]));
        acc[3] = fmaf(s_r8, C[3], fmaf(b_r8, cx.w, acc[3]));
      }
    }
    __syncwarp();
    if (lane == 0 && u + kStages < u1) {
      issue_unit(a, it, ib, smem_u32(my_ring + slot_i * kSlotBytes), smem_u32(&my_bars[slot_i]));
      if (++ib == nblk) { ib = 0; ++it; }
    }
    if (u + 1 >= u1 || blk + 1 == nblk) {
      // ---- finish this warp's share of the tile (16 rows × up to 8 x rows) ----
      const uint32_t u_first = (uint32_t)tile * (uint32_t)nblk;
      const int w_first = warp_of_unit(u_first, units, tw);
      const int w_last = warp_of_unit(u_first + nblk - 1, units, tw);
      const int nc = w_last - w_first + 1;
      const int64_t row0 = (int64_t)tile * kTileRows;
      if (nc == 1) {
        const int rr[4] = {r, r, r + 8, r + 8}, nn[4] = {n0, n1, n0, n1};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (nn[q] < R && row0 + rr[q] < a.N) a.y[(int64_t)nn[q] * a.N + row0 + rr[q]] = __float2half_rn(acc[q]);
      } else {
        float* p = a.partial + ((int64_t)tile * a.maxc + (gw - w_first)) * (kTileRows * kRowsMax);
        p[r * kRowsMax + n0] = acc[0];
        p[r * kRowsMax + n1] = acc[1];
        p[(r + 8) * kRowsMax + n0] = acc[2];
        p[(r + 8) * kRowsMax + n1] = acc[3];
        __syncwarp();
        int old = 0;
        if (lane == 0) {
          __threadfence();
          old = atomicAdd(a.counters + tile, 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == nc - 1) {
          __threadfence();
          const float* base = a.partial + (int64_t)tile * a.maxc * (kTileRows * kRowsMax);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int idx = lane * 4 + q, row = idx / kRowsMax, n = idx % kRowsMax;
            float sum = 0.f;
            for (int i = 0; i < nc; ++i) sum += __ldcg(base + i * (kTileRows * kRowsMax) + idx);
            if (n < R && row0 + row < a.N) a.y[(int64_t)n * a.N + row0 + row] = __float2half_rn(sum);
          }
          // leave the partial region zero: the one-row kernels' reduction shares it
          float* clr = a.partial + (int64_t)tile * a.maxc * (kTileRows * kRowsMax);
          for (int i = 0; i < nc; ++i) {
#pragma unroll
            for (int q = 0; q < 4; ++q) clr[i * (kTileRows * kRowsMax) + lane * 4 + q] = 0.f;
          }
          if (lane == 0) a.counters[tile] = 0;
        }
      }
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
    if (++blk == nblk) { blk = 0; ++tile; }
  }
  if (!ok && lane == 0 && a.err) atomicExch(a.err, 1);
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

struct Plan {
  int ctas;
  int total_warps;
  int64_t units;
  int nblk, ntiles, maxc;
  size_t smem;
  size_t ws_partial;  // bytes
  size_t ws_counters;
};

int g_num_sms = 0;

int num_sms() {
  if (!g_num_sms) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
      g_num_sms = n;
    else
      g_num_sms = 148;
  }
  return g_num_sms;
}

Plan make_plan(int64_t N, int64_t K, int sms, int warps_per_cta) {
  Plan p;
  p.nblk = (int)ceil_div(K, kBlockK);
  p.ntiles = (int)ceil_div(N, kTileRows);
  p.units = (int64_t)p.ntiles * p.nblk;
  int64_t ctas = sms;
  if (ctas * warps_per_cta > p.units) ctas = ceil_div(p.units, warps_per_cta);
  p.ctas = (int)(ctas < 1 ? 1 : ctas);
  // With fewer units than warps, each working warp takes exactly one unit and the
  // surplus warps (gw >= total_warps) stay idle, so every counted warp contributes.
  p.total_warps = (int)(p.units < (int64_t)p.ctas * warps_per_cta ? p.units : (int64_t)p.ctas * warps_per_cta);
  // Contributors per tile: a tile of nblk units meets at most ceil(nblk / min_units) + 1 warps.
  const int64_t min_units = p.units / p.total_warps;
  p.maxc = min_units > 0 ? (int)(ceil_div(p.nblk, min_units) + 1) : p.nblk + 1;
  if (p.maxc > p.nblk + 1) p.maxc = p.nblk + 1;
  p.smem = (size_t)K * sizeof(__half) + (size_t)(K / 64) * sizeof(float) + 32 * 3 * sizeof(float);
  p.ws_partial = sizeof(long long) * (size_t)p.ntiles * p.maxc * kTileRows;
  p.ws_counters = sizeof(int) * (size_t)p.ntiles;
  return p;
}

size_t plan_ws_bytes(const Plan& p) { return kCounterBytes + p.ws_partial; }

bool fast_path_ok(int dtype, int bits, int gs, int64_t K, const void* x, const void* w,
                  const void* sc, const void* bi) {
  auto al = [](const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
  return dtype == MOTIF_F16 && bits == 4 && gs == 64 && K % 128 == 0 && K <= 16384 && (!x || al(x, 16)) &&
         al(w, 16) && al(sc, 4) && al(bi, 4);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2D byte view (rows × inner_bytes, row pitch inner_bytes) with a box of box_rows × box_inner.
bool encode_rows(CUtensorMap* m, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_inner,
                 uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner_bytes, rows};
  cuuint64_t strides[1] = {inner_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t tma_smem_bytes(int64_t K, bool tp_in = false) {
  return (size_t)kTmaWarps * kStages * kSlotBytes + (size_t)kTmaWarps * kStages * 8 +
         (size_t)(K / 64) * kXGroupBytes + 64 + kZeroBytes + 2 * (size_t)(K / 64) * 4 + 32 * 3 * 4 +
         (tp_in ? (size_t)K * 2 : 0);
}

// The TMA kernel needs K % 512 == 0 and 16-byte aligned rows of codes (K/2 bytes) and scales (K/32 bytes).
bool try_tma(LinArgs& a) {
  if (a.K % 512 || tma_smem_bytes(a.K, a.tp_in != nullptr) > (size_t)kTmaSmemCap) return false;
  if ((reinterpret_cast<uintptr_t>(a.w) | reinterpret_cast<uintptr_t>(a.sc) | reinterpret_cast<uintptr_t>(a.bi)) % 16)
    return false;
  return encode_rows(&a.tm_w, a.w, (uint64_t)a.K / 2, (uint64_t)a.N, 128, kTileRows, CU_TENSOR_MAP_SWIZZLE_128B) &&
         encode_rows(&a.tm_s, a.sc, (uint64_t)a.K / 32, (uint64_t)a.N, 16, kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE) &&
         encode_rows(&a.tm_b, a.bi, (uint64_t)a.K / 32, (uint64_t)a.N, 16, kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Workspace bytes for shape (n, k): the larger of the two kernels' plans.
size_t ws_bytes_for(int64_t n, int64_t k) {
  const int sms = num_sms();
  const Plan p8 = make_plan(n, k, sms, kWarps);
  const Plan p16 = make_plan(n, k, sms, kTmaWarps);
  size_t b = 0;
  if (p8.units > p8.ntiles) b = plan_ws_bytes(p8);
  if (k % 512 == 0 && p16.units > p16.ntiles && plan_ws_bytes(p16) > b) b = plan_ws_bytes(p16);
  return b;
}

int launch_q4(LinArgs& a, void* workspace, size_t ws_bytes, cudaStream_t st) {
  const bool tma = try_tma(a);
  const Plan p = make_plan(a.N, a.K, num_sms(), tma ? kTmaWarps : kWarps);
  if ((uint64_t)p.units * (uint64_t)p.total_warps >= (1ull << 32))
    return fail(MOTIF_ERR_BAD_SHAPE, "quantized_linear: %lld x %lld too large", (long long)a.N, (long long)a.K);
  a.nblk = p.nblk;
  a.ntiles = p.ntiles;
  a.units = p.units;
  a.total_warps = p.total_warps;
  a.maxc = p.maxc;
  a.err = nullptr;
  if (p.units > p.ntiles) {  // some tile may be split across warps
    const size_t need = plan_ws_bytes(p);
    if (!workspace || ws_bytes < need)
      return fail(MOTIF_ERR_WORKSPACE, "quantized_linear: workspace %zu < %zu bytes", ws_bytes, need);
    if (p.ntiles > kTileCounterCap)
      return fail(MOTIF_ERR_BAD_SHAPE, "quantized_linear: n=%lld rows exceed %lld", (long long)a.N,
                  (long long)(kTileCounterCap * kTileRows));
    a.counters = static_cast<int*>(workspace);
    a.ppair = reinterpret_cast<long long*>(static_cast<char*>(workspace) + kCounterBytes);
    a.err = a.counters + kErrSlot;
  } else {
    a.counters = nullptr;
    a.ppair = nullptr;
  }
  if (a.argmax_out || a.argmax_key_out) {  // the argmax state lives in the workspace's control words
    if (!workspace || ws_bytes < kCounterBytes)
      return fail(MOTIF_ERR_WORKSPACE, "linear_fused: argmax needs a workspace of >= %zu bytes", kCounterBytes);
    int* ctl = static_cast<int*>(workspace);
    a.amax_key = reinterpret_cast<unsigned long long*>(ctl + kAmaxKeySlot);
    a.amax_tiles = ctl + kAmaxTilesSlot;
  }
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaSuccess;
    for (auto k : {q4_gemv_kernel<0>, q4_gemv_kernel<1>, q4_gemv_kernel<2>})
      if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    for (auto k : {q4_gemv_tma_kernel<0>, q4_gemv_tma_kernel<1>, q4_gemv_tma_kernel<2>})
      if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsSmemCap);
    if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "quantized_linear: smem attribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  const int64_t max_k = 8LL * 256 * (a.mode == kModeAddRms ? StageWords<1>::value : StageWords<0>::value);
  if (a.K > max_k)
    return fail(MOTIF_ERR_BAD_SHAPE, "quantized_linear: K=%lld exceeds %lld for prologue mode %d", (long long)a.K,
                (long long)max_k, a.mode);
  if (!tma && p.smem + (a.tp_in ? (size_t)a.K * 2 : 0) > 160 * 1024)
    return fail(MOTIF_ERR_BAD_SHAPE, "quantized_linear: K=%lld too large", (long long)a.K);
  if (a.tp_world) {  // the exchange waits report through the workspace's error word
    if (!workspace || ws_bytes < kCounterBytes)
      return fail(MOTIF_ERR_WORKSPACE, "linear_fused: tensor-parallel exchange needs a workspace of >= %zu bytes",
                  kCounterBytes);
    a.err = static_cast<int*>(workspace) + kErrSlot;
    a.tp_wait_ns = reinterpret_cast<unsigned long long*>(static_cast<int*>(workspace) + kTpWaitSlot);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ctas);
  cfg.blockDim = dim3(tma ? kTmaThreads : kThreads);
  cfg.dynamicSmemBytes = tma ? tma_smem_bytes(a.K, a.tp_in != nullptr) : p.smem + (a.tp_in ? (size_t)a.K * 2 : 0);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (a.mode) {
    case kModeX: e = tma ? cudaLaunchKernelEx(&cfg, q4_gemv_tma_kernel<0>, a) : cudaLaunchKernelEx(&cfg, q4_gemv_kernel<0>, a); break;
    case kModeAddRms: e = tma ? cudaLaunchKernelEx(&cfg, q4_gemv_tma_kernel<1>, a) : cudaLaunchKernelEx(&cfg, q4_gemv_kernel<1>, a); break;
    default: e = tma ? cudaLaunchKernelEx(&cfg, q4_gemv_tma_kernel<2>, a) : cudaLaunchKernelEx(&cfg, q4_gemv_kernel<2>, a); break;
  }
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "quantized_linear launch: %s", cudaGetErrorString(e));
  return check_launch("quantized_linear");
}

// Workspace of the multi-row GEMV for (n, k, rows), 0 when its shape does not fit it.
size_t rows_ws_bytes(int64_t n, int64_t k, int rows) {
  if (rows < 2 || rows > kRowsMax || k % 512 != 0) return 0;
  const int warps = rows_warps(k, rows);
  if (warps < 4) return 0;
  const Plan p = make_plan(n, k, num_sms(), warps);
  return kCounterBytes + sizeof(float) * (size_t)p.ntiles * p.maxc * kTileRows * kRowsMax;
}

// Most x rows one launch stages for in-dimension k (at least 4 warps of ring beside them), 0 if
// not even two fit.
int rows_cap(int64_t k) {
  if (k % 512) return 0;
  for (int r = kRowsMax; r >= 2; --r)
    if (rows_warps(k, r) >= 4) return r;
  return 0;
}

// Workspace for m rows taken in balanced chunks of up to rows_cap(k) rows (sizes q and q + 1; a
// one-row chunk runs the one-row kernel), 0 if the multi-row kernel does not fit.
size_t rows_ws_need(int64_t n, int64_t k, int64_t m) {
  const int cap = rows_cap(k);
  if (!cap || m < 2) return 0;
  const int64_t chunks = ceil_div(m, cap);
  const int q = (int)(m / chunks);
  auto need = [&](int rows) { return rows == 1 ? ws_bytes_for(n, k) : rows_ws_bytes(n, k, rows); };
  const size_t a = need(q);
  const size_t b = m % chunks ? need(q + 1) : a;
  return a > b ? a : b;
}

// y (rows, n) = x (rows, k) · dequant(W)ᵀ with the weights streamed once; returns -1 (nothing
// launched) when the shape or the workspace does not fit the kernel.
int launch_q4_rows(LinArgs& a, int rows, void* workspace, size_t ws_bytes, cudaStream_t st) {
  const size_t need = rows_ws_bytes(a.N, a.K, rows);
  if (!need || !workspace || ws_bytes < need || !try_tma(a)) return -1;
  const int warps = rows_warps(a.K, rows);
  const Plan p = make_plan(a.N, a.K, num_sms(), warps);
  if ((uint64_t)p.units * (uint64_t)p.total_warps >= (1ull << 32) || p.ntiles > kTileCounterCap) return -1;
  a.nblk = p.nblk;
  a.ntiles = p.ntiles;
  a.units = p.units;
  a.total_warps = p.total_warps;
  a.maxc = p.maxc;
  a.counters = static_cast<int*>(workspace);
  a.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  a.err = a.counters + kErrSlot;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaSuccess;
    for (auto k : {q4_gemv_rows_kernel<2>, q4_gemv_rows_kernel<3>, q4_gemv_rows_kernel<4>, q4_gemv_rows_kernel<5>,
                   q4_gemv_rows_kernel<6>, q4_gemv_rows_kernel<7>, q4_gemv_rows_kernel<8>})
      if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsSmemCap);
    if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "quantized_linear rows: smem attribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ctas);
  cfg.blockDim = dim3(warps * 32);
  cfg.dynamicSmemBytes = rows_smem_bytes(a.K, rows, warps);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (rows) {
    case 2: e = cudaLaunchKernelEx(&cfg, q4_gemv_rows_kernel<2>, a); break;
    case 3: e = cudaLaunchKernelEx(&cfg, q4_gemv_rows_kernel<3>, a); break;
    case 4: e = cudaLaunchKernelEx(&cfg, q4_gemv_rows_kernel<4>, a); break;
    case 5: e = cudaLaunchKernelEx(&cfg, q4_gemv_rows_kernel<5>, a); break;
    case 6: e = cudaLaunchKernelEx(&cfg, q4_gemv_rows_kernel<6>, a); break;
    case 7: e = cudaLaunchKernelEx(&cfg, q4_gemv_rows_kernel<7>, a); break;
    default: e = cudaLaunchKernelEx(&cfg, q4_gemv_rows_kernel<8>, a); break;
  }
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "quantized_linear rows launch: %s", cudaGetErrorString(e));
  return check_launch("quantized_linear rows");
}

bool al16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % 16) == 0; }

}  // namespace

bool q4_gemm_supported(int dtype, int bits, int group_size, int64_t m, int64_t n, int64_t k, const void* x,
                       const void* w, const void* sc, const void* bi, const void* y);
int q4_gemm(const void* x, int64_t m, int64_t k, const uint32_t* w, const void* scales, const void* biases, int64_t n,
            void* y, const void* residual, int* err, cudaStream_t st);

bool encode_tma_rows(CUtensorMap* m, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_inner,
                     uint32_t box_rows, bool swizzle128) {
  return encode_rows(m, base, inner_bytes, rows, box_inner, box_rows,
                     swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace motif

using namespace motif;

extern "C" {

size_t motif_quantized_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int bits,
                                              int group_size) {
  if (bits != 4 || group_size != 64 || k % 128 != 0 || n <= 0) return 0;
  const size_t one = ws_bytes_for(n, k);
  const size_t rows = rows_ws_need(n, k, m);
  return rows > one ? rows : one;
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
  // prompt-length inputs: the tcgen05 GEMM (dequantized weight tiles on the tensor cores)
  if (q4_gemm_supported(dtype, bits, group_size, m, n, k, x, w, scales, biases, y))
    return q4_gemm(x, m, k, w, scales, biases, n, y, nullptr, nullptr, st);
  if (fast_path_ok(dtype, bits, group_size, k, x, w, scales, biases)) {
    // several rows: balanced chunks of up to kRowsMax rows, each streaming the weights once
    const size_t rows_need = rows_ws_need(n, k, m);
    if (rows_need && workspace && workspace_bytes >= rows_need) {
      const int64_t chunks = ceil_div(m, rows_cap(k));
      int64_t row = 0;
      for (int64_t i = 0; i < chunks; ++i) {
        const int rows = (int)(m / chunks + (i < m % chunks ? 1 : 0));
        LinArgs a{};
        a.w = w;
        a.sc = static_cast<const __half*>(scales);
        a.bi = static_cast<const __half*>(biases);
        a.N = n;
        a.K = k;
        a.y = static_cast<__half*>(y) + row * n;
        a.mode = kModeX;
        a.x = static_cast<const __half*>(x) + row * k;
        const int rc = rows == 1 ? launch_q4(a, workspace, workspace_bytes, st)
                                 : launch_q4_rows(a, rows, workspace, workspace_bytes, st);
        if (rc < 0 && row == 0) break;  // the weights' tensor maps could not be encoded: one row at a time
        if (rc < 0) return fail(MOTIF_ERR_CUDA, "quantized_linear rows: chunk %lld not launched", (long long)i);
        if (rc) return rc;
        row += rows;
      }
      if (row == m) return MOTIF_OK;
    }
    // Shapes the multi-row kernel does not take (k not a multiple of 512, as the o and down
    // shards of an 8-way tensor-parallel split): a few rows run the one-row GEMV each; a longer
    // block runs the general kernel below in one launch instead of one launch per row.
    if (m <= 4 || rows_need) {
      for (int64_t i = 0; i < m; ++i) {
        LinArgs a{};
        a.w = w;
        a.sc = static_cast<const __half*>(scales);
        a.bi = static_cast<const __half*>(biases);
        a.N = n;
        a.K = k;
        a.y = static_cast<__half*>(y) + i * n;
        a.mode = kModeX;
        a.x = static_cast<const __half*>(x) + i * k;
        int rc = launch_q4(a, workspace, workspace_bytes, st);
        if (rc) return rc;
      }
      return MOTIF_OK;
    }
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

size_t motif_linear_fused_workspace_bytes(int64_t n, int64_t k) {
  const size_t b = motif_quantized_linear_workspace_bytes(1, n, k, 4, 64);
  return b > kCounterBytes ? b : kCounterBytes;  // the control words (argmax state) always fit
}

int motif_linear_fused(const motif_linear_io* io, const uint32_t* w, const void* scales,
                       const void* biases, int64_t n, int64_t k, void* y, void* workspace,
                       size_t workspace_bytes, void* stream) {
  MOTIF_REQUIRE(io && w && scales && biases && y, MOTIF_ERR_NULL, "linear_fused: null pointer");
  MOTIF_REQUIRE(n > 0 && k > 0 && k % 128 == 0 && k <= 65536, MOTIF_ERR_BAD_SHAPE,
                "linear_fused: n=%lld k=%lld (k must be a multiple of 128)", (long long)n, (long long)k);
  MOTIF_REQUIRE(fast_path_ok(MOTIF_F16, 4, 64, k, nullptr, w, scales, biases), MOTIF_ERR_BAD_SHAPE,
                "linear_fused: misaligned weights");
  LinArgs a{};
  a.w = w;
  a.sc = static_cast<const __half*>(scales);
  a.bi = static_cast<const __half*>(biases);
  a.N = n;
  a.K = k;
  a.y = static_cast<__half*>(y);
  a.mode = io->mode;
  switch (io->mode) {
    case kModeX:
      MOTIF_REQUIRE(io->x && al16(io->x), MOTIF_ERR_NULL, "linear_fused: mode 0 needs a 16-byte aligned x");
      a.x = static_cast<const __half*>(io->x);
      break;
    case kModeAddRms:
      MOTIF_REQUIRE((io->h_in || (io->token && io->embed)) && io->norm_w, MOTIF_ERR_NULL,
                    "linear_fused: mode 1 needs h_in (or token+embed) and norm_w");
      MOTIF_REQUIRE(al16(io->h_in) && al16(io->embed) && al16(io->delta) && al16(io->h_out) && al16(io->norm_w),
                    MOTIF_ERR_BAD_SHAPE, "linear_fused: mode 1 vectors must be 16-byte aligned");
      a.h_in = static_cast<const __half*>(io->h_in);
      a.token = io->token;
      a.embed = static_cast<const __half*>(io->embed);
      a.vocab = io->vocab;
      a.delta = static_cast<const __half*>(io->delta);
      a.h_out = static_cast<__half*>(io->h_out);
      a.norm_w = static_cast<const __half*>(io->norm_w);
      a.eps = io->eps;
      break;
    case kModePoly:
      MOTIF_REQUIRE(io->gate && io->up && io->stats && io->stats_count > 0 && io->poly_w && io->poly_b &&
                        io->poly_dim > 0,
                    MOTIF_ERR_NULL, "linear_fused: mode 2 needs gate, up, stats, polynorm weight/bias");
      MOTIF_REQUIRE(al16(io->gate) && al16(io->up), MOTIF_ERR_BAD_SHAPE, "linear_fused: gate/up must be 16-byte aligned");
      a.gate = static_cast<const __half*>(io->gate);
      a.up = static_cast<const __half*>(io->up);
      a.stats = io->stats;
      a.stats_count = (int)io->stats_count;
      a.poly_w = static_cast<const __half*>(io->poly_w);
      a.poly_b = static_cast<const __half*>(io->poly_b);
      a.poly_eps = io->poly_eps;
      a.poly_inv_dim = 1.0f / (float)io->poly_dim;
      break;
    default:
      return fail(MOTIF_ERR_BAD_SHAPE, "linear_fused: mode %d not in {0,1,2}", io->mode);
  }
  MOTIF_REQUIRE(!io->pos_len_inc || io->argmax_out, MOTIF_ERR_BAD_CONTRACT, "linear_fused: pos_len_inc needs argmax_out");
  MOTIF_REQUIRE(io->argmax_row_offset >= 0 && io->argmax_row_offset + n <= 0xFFFFFFFFll, MOTIF_ERR_BAD_SHAPE,
                "linear_fused: argmax rows must fit 32 bits");
  a.argmax_out = io->argmax_out;
  a.pos_len_inc = io->pos_len_inc;
  a.argmax_key_out = reinterpret_cast<long long*>(io->argmax_key_out);
  a.argmax_row_offset = io->argmax_row_offset;
  if (io->tp_world) {
    MOTIF_REQUIRE(io->tp_world >= 1 && io->tp_world <= 8 && io->tp_seq && io->tp_tag >= 0 && io->tp_tag < 1024,
                  MOTIF_ERR_BAD_CONTRACT, "linear_fused: tp_world %d (1..8) needs tp_seq, tp_tag %d (0..1023)",
                  io->tp_world, io->tp_tag);
    MOTIF_REQUIRE(!io->tp_in || io->mode == kModeAddRms, MOTIF_ERR_BAD_CONTRACT, "linear_fused: tp_in needs mode 1");
    MOTIF_REQUIRE(!io->tp_in || !io->delta, MOTIF_ERR_BAD_CONTRACT, "linear_fused: tp_in replaces delta");
    MOTIF_REQUIRE(!io->tp_stats_in || io->mode == kModePoly, MOTIF_ERR_BAD_CONTRACT,
                  "linear_fused: tp_stats_in needs mode 2");
    MOTIF_REQUIRE(!io->tp_stats[0] || (io->stats_rows > 0 && io->stats_rows % kTileRows == 0 && io->stats_rows <= n),
                  MOTIF_ERR_BAD_SHAPE, "linear_fused: tp_stats needs stats_rows");
    for (int r = 0; r < io->tp_world; ++r)
      MOTIF_REQUIRE((!io->tp_out[0] || io->tp_out[r]) && (!io->tp_stats[0] || io->tp_stats[r]), MOTIF_ERR_NULL,
                    "linear_fused: tp_out/tp_stats of rank %d", r);
    a.tp_world = io->tp_world;
    a.tp_seq = io->tp_seq;
    a.tp_tag = io->tp_tag;
    for (int r = 0; r < 8; ++r) {
      a.tp_out[r] = reinterpret_cast<long long*>(io->tp_out[r]);
      a.tp_stats[r] = reinterpret_cast<long long*>(io->tp_stats[r]);
    }
    a.tp_in = reinterpret_cast<const long long*>(io->tp_in);
    a.tp_stats_in = reinterpret_cast<const long long*>(io->tp_stats_in);
    if (io->tp_stats[0] && !io->stats_out) a.stats_rows = io->stats_rows;
  }
  if (io->stats_out) {
    MOTIF_REQUIRE(io->stats_rows > 0 && io->stats_rows % kTileRows == 0 && io->stats_rows <= n, MOTIF_ERR_BAD_SHAPE,
                  "linear_fused: stats_rows must be a positive multiple of 16 and <= n");
    a.stats_out = io->stats_out;
    a.stats_rows = io->stats_rows;
  }
  return launch_q4(a, workspace, workspace_bytes, as_stream(stream));
}

}  // extern "C"
