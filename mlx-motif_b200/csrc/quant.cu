// Affine group quantization (MLX layout), the 4-slot KV-cache writes and RoPE.
//
// Quantization is bit-exact to the CPU restatement (oracle.quantize): every
// step is an explicitly rounded IEEE fp32 operation (__fsub_rn / __fdiv_rn)
// so no contraction can change a code, and round() is half-away-from-zero.
//
// Thread layout for quantization: each thread owns 8 consecutive channels
// (one packed word at 4 bits, two at 8 bits); the gs/8 threads of one group
// are consecutive lanes and reduce min/max with xor-shuffles.
#include "common.cuh"
#include "kvquant.cuh"

namespace motif {
namespace {

// Maps a logical input row to its source pointer and its destination row.
struct RowMap {
  // Plain (rows, dim) input/output.
  const void* src;
  int64_t src_row_stride;
  // 4-slot mode: the input is four (B, H, S, D) tensors, the output the slots.
  bool kv4;
  const void* kv_src[4];
  uint32_t* kv_data[4];
  void* kv_scales[4];
  void* kv_biases[4];
  int64_t H, S, cap;
  const int32_t* off_dev;
  int64_t off;
  // Plain output.
  uint32_t* data;
  void* scales;
  void* biases;
};

template <typename T, int LPG>
__global__ void quantize_kernel(RowMap m, int bits, int gs, int64_t rows, int dim) {
  const int64_t chunks_per_row = dim / 8;
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = c < rows * chunks_per_row;
  const int64_t row = active ? c / chunks_per_row : 0;
  const int ch0 = active ? (int)(c - row * chunks_per_row) * 8 : 0;
  const T* src;
  uint32_t* data;
  T* scales;
  T* biases;
  int64_t out_row;
  if (m.kv4) {
    const int64_t per_slot = rows / 4;
    const int slot = (int)(row / per_slot);
    const int64_t r = row - slot * per_slot;  // (b, h, s) flattened
    const int64_t s = r % m.S;
    const int64_t bh = r / m.S;
    const int64_t off = m.off_dev ? (int64_t)*m.off_dev : m.off;
    src = static_cast<const T*>(m.kv_src[slot]) + r * dim;
    out_row = bh * m.cap + off + s;
    data = m.kv_data[slot];
    scales = static_cast<T*>(m.kv_scales[slot]);
    biases = static_cast<T*>(m.kv_biases[slot]);
  } else {
    src = static_cast<const T*>(m.src) + row * m.src_row_stride;
    out_row = row;
    data = m.data;
    scales = static_cast<T*>(m.scales);
    biases = static_cast<T*>(m.biases);
  }
  float v[8];
  if (active) {
    load_vec<T, 8>(src + ch0, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
  }
  uint32_t words[2];
  float sc, bi;
  quant_group<LPG>(v, bits, words, sc, bi);
  if (!active) return;
  const int el = 32 / bits;
  const int64_t wpr = dim / el;
  uint32_t* drow = data + out_row * wpr + ch0 / el;
  drow[0] = words[0];
  if (bits == 8) drow[1] = words[1];
  if ((ch0 % gs) == 0) {
    const int64_t g = out_row * (dim / gs) + ch0 / gs;
    scales[g] = from_f<T>(sc);
    biases[g] = from_f<T>(bi);
  }
}

template <typename T>
int launch_quantize(const RowMap& m, int bits, int gs, int64_t rows, int64_t dim, cudaStream_t st) {
  const int64_t chunks = rows * (dim / 8);
  const int threads = 256;
  const int64_t blocks = ceil_div(chunks, threads);
  switch (gs) {
    case 32: quantize_kernel<T, 4><<<blocks, threads, 0, st>>>(m, bits, gs, rows, (int)dim); break;
    case 64: quantize_kernel<T, 8><<<blocks, threads, 0, st>>>(m, bits, gs, rows, (int)dim); break;
    case 128: quantize_kernel<T, 16><<<blocks, threads, 0, st>>>(m, bits, gs, rows, (int)dim); break;
    default: return fail(MOTIF_ERR_BAD_CONTRACT, "quantize: group_size %d not in {32,64,128}", gs);
  }
  return check_launch("quantize");
}

// ---- dequantize: one thread per packed word ---------------------------------
template <typename T>
__global__ void dequantize_kernel(const uint32_t* __restrict__ data, const T* __restrict__ scales,
                                  const T* __restrict__ biases, int bits, int gs, int64_t rows,
                                  int dim, T* __restrict__ y) {
  const int el = 32 / bits;
  const int64_t wpr = dim / el;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * wpr) return;
  const int64_t row = i / wpr;
  const int w = (int)(i - row * wpr);
  const int ch0 = w * el;
  const int64_t g = row * (dim / gs) + ch0 / gs;
  const float s = to_f<T>(scales[g]);
  const float b = to_f<T>(biases[g]);
  const uint32_t word = data[i];
  const uint32_t mask = (1u << bits) - 1u;
  T* out = y + row * dim + ch0;
  for (int j = 0; j < el; ++j) {
    const float raw = (float)((word >> (j * bits)) & mask);
    out[j] = from_f<T>(__fadd_rn(__fmul_rn(s, raw), b));
  }
}

// ---- fp16 4-slot append: one thread per 16-byte chunk ------------------------
template <typename T>
__global__ void kv4_copy_kernel(const T* __restrict__ s0, const T* __restrict__ s1,
                                const T* __restrict__ s2, const T* __restrict__ s3, T* d0, T* d1,
                                T* d2, T* d3, int64_t H_S, int64_t S, int64_t cap, int D,
                                const int32_t* __restrict__ off_dev, int64_t off_host,
                                int64_t chunks_per_tensor) {
  constexpr int V = 16 / sizeof(T);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 4 * chunks_per_tensor) return;
  const int slot = (int)(i / chunks_per_tensor);
  const int64_t j = i - slot * chunks_per_tensor;
  const int64_t e = j * V;  // element index in (B, H, S, D)
  const int64_t row = e / D;
  const int c = (int)(e - row * D);
  const int64_t s = row % S;
  const int64_t bh = row / S;
  const int64_t off = off_dev ? (int64_t)*off_dev : off_host;
  const T* src = slot == 0 ? s0 : slot == 1 ? s1 : slot == 2 ? s2 : s3;
  T* dst = slot == 0 ? d0 : slot == 1 ? d1 : slot == 2 ? d2 : d3;
  *reinterpret_cast<uint4*>(dst + (bh * cap + off + s) * D + c) =
      *reinterpret_cast<const uint4*>(src + e);
  (void)H_S;
}

// ---- RoPE (non-traditional): pairs (i, i + D/2) ------------------------------
template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, int64_t rows, int S, int D,
                            const int32_t* __restrict__ off_dev, int64_t off_host,
                            const float* __restrict__ inv_freq, T* __restrict__ y) {
  const int half = D / 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * half) return;
  const int64_t row = i / half;
  const int k = (int)(i - row * half);
  const int64_t s = row % S;
  const int64_t off = off_dev ? (int64_t)*off_dev : off_host;
  const float theta = __fmul_rn((float)(off + s), inv_freq[k]);
  float sn, cs;
  sincosf(theta, &sn, &cs);
  const float x1 = to_f<T>(x[row * D + k]);
  const float x2 = to_f<T>(x[row * D + k + half]);
  y[row * D + k] = from_f<T>(__fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn)));
  y[row * D + k + half] = from_f<T>(__fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs)));
}

// ---- RoPE(q), RoPE(k), 4-slot append ------------------------------------------
// One CTA per (head, row) of the fused qkv rows: [q heads | k heads (k1,k2 pairs) |
// v heads (v1,v2 pairs)]. D threads per CTA, thread c owns channel c. Row s sits at
// position pos0 + s (pos0 = *pos_dev when given); q is written head-major (q_heads, seq, D),
// which for one row is the plain (q_heads, D) of the decode step.
template <int D, int LPG>
__global__ void rope_qkv_append_kernel(const __half* __restrict__ qkv,
                                       const float* __restrict__ inv_freq, int q_heads,
                                       int kv2, motif_kv4_slots cache,
                                       const int32_t* __restrict__ pos_dev, int64_t pos_host, int seq,
                                       int64_t qkv_stride, __half* __restrict__ q_out) {
  __shared__ float vals[D];
  pdl_trigger();
  const int head = blockIdx.x;
  const int srow = blockIdx.y;
  const int c = threadIdx.x;
  const int half = D / 2;
  const int pos = (pos_dev ? *pos_dev : (int)pos_host) + srow;
  const __half* src = qkv + srow * qkv_stride + (int64_t)head * D;
  const bool is_q = head < q_heads;
  const bool is_k = !is_q && head < q_heads + 2 * kv2;
  float v;
  if (is_q || is_k) {
    v = rope_channel(src, c, half, pos, inv_freq);
  } else {
    v = __half2float(src[c]);
  }
  const __half hv = __float2half_rn(v);
  if (is_q) {
    q_out[((int64_t)head * seq + srow) * D + c] = hv;
    return;
  }
  const int kvh = is_k ? head - q_heads : head - q_heads - 2 * kv2;
  const int slot = (is_k ? 0 : 2) + (kvh & 1);
  const int j = kvh >> 1;
  if (pos < 0 || pos >= cache.capacity) return;  // caller guarantees capacity
  const int64_t row = (int64_t)j * cache.capacity + pos;
  if (cache.bits == 16) {
    static_cast<__half*>(cache.data[slot])[row * D + c] = hv;
    return;
  }
  vals[c] = __half2float(hv);
  __syncthreads();
  if (c < 32) {  // D/8 <= 32 lanes quantize 8 channels each
    const bool act = c < D / 8;
    float x8[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) x8[t] = act ? vals[c * 8 + t] : 0.f;
    uint32_t words[2];
    float sc, bi;
    quant_group<LPG>(x8, cache.bits, words, sc, bi);
    if (act) {
      const int el = 32 / cache.bits;
      uint32_t* d = static_cast<uint32_t*>(cache.data[slot]) + row * (D / el) + (c * 8) / el;
      d[0] = words[0];
      if (cache.bits == 8) d[1] = words[1];
      const int gs = cache.group_size;
      if (((c * 8) % gs) == 0) {
        const int64_t g = row * (D / gs) + (c * 8) / gs;
        static_cast<__half*>(cache.scales[slot])[g] = __float2half_rn(sc);
        static_cast<__half*>(cache.biases[slot])[g] = __float2half_rn(bi);
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace motif

using namespace motif;

extern "C" {

int motif_quantize(int dtype, int bits, int group_size, const void* x, int64_t rows, int64_t dim,
                   uint32_t* data, void* scales, void* biases, void* stream) {
  MOTIF_REQUIRE(x && data && scales && biases, MOTIF_ERR_NULL, "quantize: null pointer");
  MOTIF_REQUIRE(bits == 4 || bits == 8, MOTIF_ERR_DTYPE, "quantize: bits=%d not in {4,8}", bits);
  MOTIF_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, MOTIF_ERR_BAD_CONTRACT,
                "quantize: group_size=%d not in {32,64,128}", group_size);
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim % group_size == 0 && dim < (1ll << 31),
                MOTIF_ERR_BAD_SHAPE, "quantize: dim=%lld must be a multiple of group_size=%d",
                (long long)dim, group_size);
  MOTIF_REQUIRE(aligned16(x), MOTIF_ERR_BAD_SHAPE, "quantize: input must be 16-byte aligned");
  if (rows == 0) return MOTIF_OK;
  RowMap m{};
  m.src = x;
  m.src_row_stride = dim;
  m.kv4 = false;
  m.data = data;
  m.scales = scales;
  m.biases = biases;
  cudaStream_t st = as_stream(stream);
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_quantize<T>(m, bits, group_size, rows, dim, st));
  return MOTIF_OK;
}

int motif_dequantize(int dtype, int bits, int group_size, const uint32_t* data,
                     const void* scales, const void* biases, int64_t rows, int64_t dim, void* y,
                     void* stream) {
  MOTIF_REQUIRE(data && scales && biases && y, MOTIF_ERR_NULL, "dequantize: null pointer");
  MOTIF_REQUIRE(bits == 4 || bits == 8, MOTIF_ERR_DTYPE, "dequantize: bits=%d not in {4,8}", bits);
  MOTIF_REQUIRE(group_size > 0 && dim % 32 == 0 && dim % group_size == 0 && group_size % (32 / bits) == 0,
                MOTIF_ERR_BAD_CONTRACT, "dequantize: need D %% 32 == 0 and D %% group_size == 0 (D=%lld, g=%d)",
                (long long)dim, group_size);
  MOTIF_REQUIRE(rows >= 0 && dim > 0 && dim < (1ll << 31), MOTIF_ERR_BAD_SHAPE, "dequantize: bad shape");
  if (rows == 0) return MOTIF_OK;
  const int64_t words = rows * (dim / (32 / bits));
  const int threads = 256;
  cudaStream_t st = as_stream(stream);
  MOTIF_DISPATCH_FLOAT(dtype, T, {
    dequantize_kernel<T><<<ceil_div(words, threads), threads, 0, st>>>(
        data, static_cast<const T*>(scales), static_cast<const T*>(biases), bits, group_size, rows,
        (int)dim, static_cast<T*>(y));
  });
  return check_launch("dequantize");
}

int motif_kv4_append(int dtype, const motif_kv4_slots* cache, const void* k1, const void* k2,
                     const void* v1, const void* v2, int64_t seq, int64_t offset,
                     const int32_t* offset_dev, void* stream) {
  MOTIF_REQUIRE(cache && k1 && k2 && v1 && v2, MOTIF_ERR_NULL, "kv4_append: null pointer");
  const motif_kv4_slots& c = *cache;
  for (int i = 0; i < 4; ++i) MOTIF_REQUIRE(c.data[i], MOTIF_ERR_NULL, "kv4_append: slot %d data is null", i);
  MOTIF_REQUIRE(c.batch > 0 && c.heads > 0 && c.capacity > 0 && c.head_dim > 0 && seq >= 0,
                MOTIF_ERR_BAD_SHAPE, "kv4_append: bad cache shape");
  MOTIF_REQUIRE(offset_dev || (offset >= 0 && offset + seq <= c.capacity), MOTIF_ERR_BAD_SHAPE,
                "kv4_append: rows [%lld, %lld) exceed capacity %lld", (long long)offset,
                (long long)(offset + seq), (long long)c.capacity);
  if (seq == 0) return MOTIF_OK;
  for (const void* p : {k1, k2, v1, v2})
    MOTIF_REQUIRE(aligned16(p), MOTIF_ERR_BAD_SHAPE, "kv4_append: inputs must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int64_t D = c.head_dim;
  if (c.bits == 16) {
    const size_t esz = dtype == MOTIF_F32 ? 4 : 2;
    MOTIF_REQUIRE((D * (int64_t)esz) % 16 == 0, MOTIF_ERR_BAD_SHAPE, "kv4_append: head_dim*esize must be a multiple of 16");
    for (int i = 0; i < 4; ++i) MOTIF_REQUIRE(aligned16(c.data[i]), MOTIF_ERR_BAD_SHAPE, "kv4_append: slot not 16-byte aligned");
    const int64_t per = c.batch * c.heads * seq * D * (int64_t)esz / 16;
    const int threads = 256;
    MOTIF_DISPATCH_FLOAT(dtype, T, {
      kv4_copy_kernel<T><<<ceil_div(4 * per, threads), threads, 0, st>>>(
          static_cast<const T*>(k1), static_cast<const T*>(k2), static_cast<const T*>(v1),
          static_cast<const T*>(v2), static_cast<T*>(c.data[0]), static_cast<T*>(c.data[1]),
          static_cast<T*>(c.data[2]), static_cast<T*>(c.data[3]), c.heads * seq, seq, c.capacity,
          (int)D, offset_dev, offset, per);
    });
    return check_launch("kv4_append");
  }
  MOTIF_REQUIRE(c.bits == 4 || c.bits == 8, MOTIF_ERR_DTYPE, "kv4_append: bits=%d not in {4,8,16}", c.bits);
  MOTIF_REQUIRE(c.group_size == 32 || c.group_size == 64 || c.group_size == 128, MOTIF_ERR_BAD_CONTRACT,
                "kv4_append: group_size %d not in {32,64,128}", c.group_size);
  MOTIF_REQUIRE(D % c.group_size == 0, MOTIF_ERR_BAD_SHAPE, "kv4_append: head_dim %% group_size != 0");
  for (int i = 0; i < 4; ++i)
    MOTIF_REQUIRE(c.scales[i] && c.biases[i], MOTIF_ERR_NULL, "kv4_append: slot %d scales/biases null", i);
  RowMap m{};
  m.kv4 = true;
  const void* srcs[4] = {k1, k2, v1, v2};
  for (int i = 0; i < 4; ++i) {
    m.kv_src[i] = srcs[i];
    m.kv_data[i] = static_cast<uint32_t*>(c.data[i]);
    m.kv_scales[i] = c.scales[i];
    m.kv_biases[i] = c.biases[i];
  }
  m.H = c.heads;
  m.S = seq;
  m.cap = c.capacity;
  m.off_dev = offset_dev;
  m.off = offset;
  const int64_t rows = 4 * c.batch * c.heads * seq;
  MOTIF_DISPATCH_FLOAT(dtype, T, return launch_quantize<T>(m, c.bits, c.group_size, rows, D, st));
  return MOTIF_OK;
}

int motif_rope(int dtype, const void* x, int64_t batch, int64_t heads, int64_t seq, int64_t dim,
               int64_t offset, const int32_t* offset_dev, const float* inv_freq, void* y,
               void* stream) {
  MOTIF_REQUIRE(x && inv_freq && y, MOTIF_ERR_NULL, "rope: null pointer");
  MOTIF_REQUIRE(batch >= 0 && heads >= 0 && seq > 0 && dim > 0 && dim % 2 == 0, MOTIF_ERR_BAD_SHAPE,
                "rope: bad shape");
  const int64_t rows = batch * heads * seq;
  if (rows == 0) return MOTIF_OK;
  const int threads = 256;
  const int64_t n = rows * (dim / 2);
  cudaStream_t st = as_stream(stream);
  MOTIF_DISPATCH_FLOAT(dtype, T, {
    rope_kernel<T><<<ceil_div(n, threads), threads, 0, st>>>(static_cast<const T*>(x), rows, (int)seq,
                                                             (int)dim, offset_dev, offset, inv_freq,
                                                             static_cast<T*>(y));
  });
  return check_launch("rope");
}

static int rope_qkv_append_launch(const void* qkv, int64_t seq, const float* inv_freq, int64_t q_heads,
                                  const motif_kv4_slots* cache, int64_t pos_host, const int32_t* pos_dev,
                                  void* q_out, void* stream) {
  MOTIF_REQUIRE(qkv && inv_freq && cache && q_out, MOTIF_ERR_NULL, "rope_qkv_append: null pointer");
  const motif_kv4_slots& c = *cache;
  MOTIF_REQUIRE(c.batch == 1 && c.head_dim == 128, MOTIF_ERR_BAD_CONTRACT,
                "rope_qkv_append: batch 1 and head_dim 128 only (got %lld, %lld)", (long long)c.batch,
                (long long)c.head_dim);
  MOTIF_REQUIRE(seq >= 1 && seq < 65536 && q_heads >= 1, MOTIF_ERR_BAD_SHAPE, "rope_qkv_append: seq=%lld",
                (long long)seq);
  MOTIF_REQUIRE(pos_dev || (pos_host >= 0 && pos_host + seq <= c.capacity), MOTIF_ERR_BAD_SHAPE,
                "rope_qkv_append: rows [%lld, %lld) outside capacity %lld", (long long)pos_host,
                (long long)(pos_host + seq), (long long)c.capacity);
  for (int i = 0; i < 4; ++i) MOTIF_REQUIRE(c.data[i], MOTIF_ERR_NULL, "rope_qkv_append: slot %d null", i);
  const dim3 grid((unsigned)(q_heads + 4 * c.heads), (unsigned)seq);
  const int64_t stride = (q_heads + 4 * c.heads) * 128;
  cudaStream_t st = as_stream(stream);
  auto qkv_p = static_cast<const __half*>(qkv);
  auto q_p = static_cast<__half*>(q_out);
  const int qh = (int)q_heads, kv2 = (int)c.heads, S = (int)seq;
  if (c.bits == 16) {
    rope_qkv_append_kernel<128, 8><<<grid, 128, 0, st>>>(qkv_p, inv_freq, qh, kv2, c, pos_dev, pos_host, S, stride, q_p);
  } else {
    MOTIF_REQUIRE(c.bits == 4 || c.bits == 8, MOTIF_ERR_DTYPE, "rope_qkv_append: bits=%d", c.bits);
    for (int i = 0; i < 4; ++i)
      MOTIF_REQUIRE(c.scales[i] && c.biases[i], MOTIF_ERR_NULL, "rope_qkv_append: slot %d scales/biases null", i);
    switch (c.group_size) {
      case 32: rope_qkv_append_kernel<128, 4><<<grid, 128, 0, st>>>(qkv_p, inv_freq, qh, kv2, c, pos_dev, pos_host, S, stride, q_p); break;
      case 64: rope_qkv_append_kernel<128, 8><<<grid, 128, 0, st>>>(qkv_p, inv_freq, qh, kv2, c, pos_dev, pos_host, S, stride, q_p); break;
      case 128: rope_qkv_append_kernel<128, 16><<<grid, 128, 0, st>>>(qkv_p, inv_freq, qh, kv2, c, pos_dev, pos_host, S, stride, q_p); break;
      default: return fail(MOTIF_ERR_BAD_CONTRACT, "rope_qkv_append: group_size %d", c.group_size);
    }
  }
  return check_launch("rope_qkv_append");
}

int motif_rope_qkv_append(const void* qkv, const float* inv_freq, int64_t q_heads,
                          const motif_kv4_slots* cache, const int32_t* pos_dev, void* q_out,
                          void* stream) {
  MOTIF_REQUIRE(pos_dev, MOTIF_ERR_NULL, "rope_qkv_append: null pointer");
  return rope_qkv_append_launch(qkv, 1, inv_freq, q_heads, cache, 0, pos_dev, q_out, stream);
}

int motif_rope_qkv_append_rows(const void* qkv, int64_t seq, const float* inv_freq, int64_t q_heads,
                               const motif_kv4_slots* cache, int64_t offset, const int32_t* offset_dev,
                               void* q_out, void* stream) {
  return rope_qkv_append_launch(qkv, seq, inv_freq, q_heads, cache, offset, offset_dev, q_out, stream);
}

}  // extern "C"
