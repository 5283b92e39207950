// Softmax row statistics in the reference operator's exact arithmetic.
//
// For one (query, group) row of logits the reference (csrc/scoring.cu:32-66)
// computes x = dtype(float(logit) * scale), masked to -inf where the key's
// position exceeds the query's; the row max; 256 per-thread sequential sums
// of expf(x - max) over positions t, t+256, ... folded by a pairwise tree
// (csrc/scoring.cu:15-30) into the denominator; p = w / denominator; and the
// same lane-order sum of p * projected_value.  Every kernel here reproduces
// those operations and their order exactly (the including file is compiled
// with --fmad=false, and order-sensitive steps use _rn intrinsics), so the
// max, denominator, projection and probabilities are bit-identical.
//
// The work is arranged for B200: one CTA of 256 threads (the 256 reference
// lanes) per row; the row is read from HBM once with 16-byte loads and staged
// in shared memory -- as fp32 weights for rows up to 18k positions (3 CTAs per
// SM; the weights are computed once and reused by pass C), in the logits dtype
// (exact) up to 110k bf16 positions -- and the reduction passes then run from
// shared memory.  Longer rows recompute x from the logits in each pass.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"

namespace lrk {
namespace rows {

constexpr int kLanes = 256;  // the reference's reduction width; one thread per lane
constexpr int kStageBytes = 220 * 1024;

template <typename T> struct Dtype;
template <> struct Dtype<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
  using Bits = unsigned short;
  static __device__ __forceinline__ float to_float(Bits b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
  static __device__ __forceinline__ Bits round(float x, float scale) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(x, scale)));
  }
};
template <> struct Dtype<__half> {
  static constexpr int kPerVec = 8;
  using Bits = unsigned short;
  static __device__ __forceinline__ float to_float(Bits b) { return __half2float(__ushort_as_half(b)); }
  static __device__ __forceinline__ Bits round(float x, float scale) {
    return __half_as_ushort(__float2half_rn(__fmul_rn(x, scale)));
  }
};
template <> struct Dtype<float> {
  static constexpr int kPerVec = 4;
  using Bits = uint32_t;
  static __device__ __forceinline__ float to_float(Bits b) { return __uint_as_float(b); }
  static __device__ __forceinline__ Bits round(float x, float scale) { return __float_as_uint(__fmul_rn(x, scale)); }
};

// -inf in each dtype's bit pattern.
template <typename T> __device__ __forceinline__ typename Dtype<T>::Bits minus_infinity();
template <> __device__ __forceinline__ unsigned short minus_infinity<__nv_bfloat16>() { return 0xff80u; }
template <> __device__ __forceinline__ unsigned short minus_infinity<__half>() { return 0xfc00u; }
template <> __device__ __forceinline__ uint32_t minus_infinity<float>() { return 0xff800000u; }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block max over NT threads (order-free); scratch holds >= 32 floats.
template <int NT = kLanes>
__device__ __forceinline__ float block_max(float v, float *scratch) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = threadIdx.x < NT / 32 ? scratch[threadIdx.x] : -INFINITY;
  if (threadIdx.x < 32) r = warp_max(r);
  if (threadIdx.x == 0) scratch[0] = r;
  __syncthreads();
  r = scratch[0];
  __syncthreads();
  return r;
}

// block_max of two values at once (one pair of barriers).
__device__ __forceinline__ float2 block_max2(float a, float b, float *scratch) {
  a = warp_max(a);
  b = warp_max(b);
  if ((threadIdx.x & 31) == 0) {
    scratch[threadIdx.x >> 5] = a;
    scratch[32 + (threadIdx.x >> 5)] = b;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    float ra = threadIdx.x < kLanes / 32 ? scratch[threadIdx.x] : -INFINITY;
    float rb = threadIdx.x < kLanes / 32 ? scratch[32 + threadIdx.x] : -INFINITY;
    ra = warp_max(ra);
    rb = warp_max(rb);
    if (threadIdx.x == 0) scratch[64] = ra, scratch[65] = rb;
  }
  __syncthreads();
  const float2 r = make_float2(scratch[64], scratch[65]);
  __syncthreads();
  return r;
}

// The reference's 256-wide pairwise tree: partial[t] += partial[t + s] for
// s = 128 .. 1.  Lanes are threads 0..255; all threads of the CTA call.  tree
// holds 256 floats.
__device__ __forceinline__ float tree_sum(float partial, float *tree) {
  if (threadIdx.x < kLanes) tree[threadIdx.x] = partial;
  __syncthreads();
#pragma unroll
  for (int s = kLanes / 2; s >= 32; s >>= 1) {
    if (threadIdx.x < s) tree[threadIdx.x] = __fadd_rn(tree[threadIdx.x], tree[threadIdx.x + s]);
    __syncthreads();
  }
  if (threadIdx.x < 32) {
    float value = tree[threadIdx.x];
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      const float other = __shfl_down_sync(0xffffffffu, value, s);
      if (threadIdx.x < s) value = __fadd_rn(value, other);
    }
    if (threadIdx.x == 0) tree[0] = value;
  }
  __syncthreads();
  const float result = tree[0];
  __syncthreads();
  return result;
}

// Correctly rounded a / b for a row's probabilities, b = the row's
// denominator (>= 1 when finite), a = an exp weight in [0, 1].  With the
// correctly rounded reciprocal y = RN(1/b), q0 = RN(a y) is within 2 ulp of
// a/b; one residual step q1 = RN(q0 + y RN(a - b q0)) makes it faithful (the
// residual is exact in one FMA), and a second step is Markstein's theorem: if y
// is within half an ulp of 1/b and q1 within one ulp of a/b, RN(q1 + y r1) is
// RN(a/b) (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; Muller et al.,
// Handbook of Floating-Point Arithmetic, 2nd ed., 2018, section 4.7).  The
// theorem needs every residual and quotient in the normal range, which
// 1 <= b <= 2^32 and 2^-60 <= a <= 2^32 guarantee; other operands (0,
// subnormal, NaN, inf) take the IEEE division itself.  Correct rounding is
// unique, so the result equals __fdiv_rn bit for bit; lrk_check_division
// tests that on the GPU.
struct Divider {
  float b, y;
  bool fast;
};

__device__ __forceinline__ Divider make_divider(float denominator) {
  Divider d;
  d.b = denominator;
  d.y = __frcp_rn(denominator);
  d.fast = denominator >= 1.0f && denominator <= 4294967296.0f;  // false for NaN
  return d;
}

__device__ __forceinline__ float divide(const Divider &d, float a) {
  if (d.fast && a >= 8.673617379884035e-19f && a <= 4294967296.0f) {  // 2^-60, 2^32
    float q = __fmul_rn(a, d.y);
    q = __fmaf_rn(__fmaf_rn(-q, d.b, a), d.y, q);
    return __fmaf_rn(__fmaf_rn(-q, d.b, a), d.y, q);
  }
  return __fdiv_rn(a, d.b);
}

struct RowResult {
  float maximum, denominator, projection;
};

// Layouts of a row between its passes (one CTA of 256 threads = the 256
// reference lanes per row).
enum Stage : int {
  kStream = 0,   // nothing staged: x is recomputed from the logits in each pass
  kBits = 1,     // x staged in the logits dtype (exact), expf recomputed in pass C
  kWeights = 2,  // x staged as fp32 and overwritten by w = expf(x - max) in pass B
  kPacked = 3,   // kBits for 16-bit logits in 16-byte aligned rows, lane-major
                 // (row_statistics_packed): 8 elements per lane per 16-byte
                 // chunk, pairs of elements in float2 arithmetic
};

template <typename T>
__host__ __device__ constexpr int64_t staged_bytes(int mode, int64_t length) {
  return mode == kWeights                    ? (length + 8) * 4
         : mode == kBits || mode == kPacked ? (length + 16) * static_cast<int64_t>(sizeof(typename Dtype<T>::Bits))
                                             : 0;
}

// Rows up to this many fp32 weights (72 KB, 3 CTAs per SM) keep w.
#ifndef LRK_WEIGHT_STAGE_MAX
#define LRK_WEIGHT_STAGE_MAX (18 * 1024)
#endif
constexpr int64_t kWeightStageMax = LRK_WEIGHT_STAGE_MAX;

// aligned: every row starts on a 16-byte boundary.
template <typename T>
inline int choose_stage(int64_t length, bool aligned) {
  constexpr bool kSixteenBit = sizeof(typename Dtype<T>::Bits) == 2;
  if (length <= kWeightStageMax) return kWeights;
  if (staged_bytes<T>(kBits, length) <= kStageBytes) return kSixteenBit && aligned ? kPacked : kBits;
  return kStream;
}

// Which keys a row sees.  The reference masks key p when key_positions[p] >
// query_position.  When the caller knows the visible keys form a prefix (key
// positions non-decreasing, as in an append-only cache), `visible` is that
// prefix's length and the mask is an index compare; visible < 0 compares
// positions element by element.
struct Visibility {
  const float *key_positions;
  float query_position;
  int64_t visible;
  __device__ __forceinline__ bool operator()(int64_t p) const {
    return visible >= 0 ? p < visible : __ldg(key_positions + p) <= query_position;
  }
  // Every key of [p, p + n) is visible (index test only).
  __device__ __forceinline__ bool all(int64_t p, int64_t n) const { return visible >= 0 && p + n <= visible; }
};

// Optional output of pass C: the probability of every candidate column
// [first, last) at out[p - first] -- the p the reference's risk starts from
// (csrc/scoring.cu:68-128), so the risk step need not recompute it from the
// logits.  Disabled when out is null.
struct CandidateOut {
  float *out;
  int64_t first, last;
  __device__ __forceinline__ bool wanted(int64_t p) const { return p >= first && p < last; }
  __device__ __forceinline__ void put(int64_t p, float probability) const { out[p - first] = probability; }
};

template <typename T>
__device__ RowResult row_statistics_packed(const T *__restrict__ row, int64_t length, const Visibility sees,
                                           const float *__restrict__ projected_values, float scale,
                                           float *__restrict__ probabilities_out, unsigned char *stage,
                                           float *scratch, const CandidateOut candidates);

// Statistics of one row (all 256 threads call).  probabilities_out, when not
// null, receives every probability (the drop-in operator's output).  `stage`
// is dynamic shared memory of staged_bytes<T>(MODE, length) bytes.  Global
// loads are issued in batches ahead of their use (kBatch vectors or elements
// per thread), which hides their latency at 3 CTAs per SM.
template <typename T, int MODE>
__device__ RowResult row_statistics(const T *__restrict__ row, int64_t length, const Visibility sees,
                                    const float *__restrict__ projected_values, float scale,
                                    float *__restrict__ probabilities_out, unsigned char *stage, float *scratch,
                                    const CandidateOut candidates = CandidateOut{nullptr, 0, 0}) {
  if constexpr (MODE == kPacked) {
    return row_statistics_packed<T>(row, length, sees, projected_values, scale, probabilities_out, stage, scratch,
                                    candidates);
  }
  using D = Dtype<T>;
  using Bits = typename D::Bits;
  constexpr int V = D::kPerVec;
  constexpr int kBatch = 8;
  const Bits *in = reinterpret_cast<const Bits *>(row);
  // First 16-byte boundary of the row, and the stage offsets that align it.
  const int64_t lead = lmin(length, static_cast<int64_t>(((16 - (reinterpret_cast<uintptr_t>(row) & 15)) & 15) /
                                                        sizeof(Bits)));
  Bits *x_bits = reinterpret_cast<Bits *>(stage) + (V - lead % V) % V;
  float *x_float = reinterpret_cast<float *>(stage) + (4 - lead % 4) % 4;
  const Bits neg_inf = minus_infinity<T>();
  auto value_bits = [&](int64_t p, Bits raw) -> Bits { return sees(p) ? D::round(D::to_float(raw), scale) : neg_inf; };

  // Pass A: scale, round, mask; row max; stage the row.
  float local_max = -INFINITY;
  if (MODE == kStream) {
    for (int64_t p = threadIdx.x; p < length; p += kLanes)
      local_max = fmaxf(local_max, D::to_float(value_bits(p, __ldg(in + p))));
  } else {
    auto put = [&](int64_t p, Bits b) {
      if (MODE == kBits) x_bits[p] = b; else x_float[p] = D::to_float(b);
      local_max = fmaxf(local_max, D::to_float(b));
    };
    for (int64_t p = threadIdx.x; p < lead; p += kLanes) put(p, value_bits(p, __ldg(in + p)));
    const int64_t vectors = (length - lead) / V;
    const uint4 *body = reinterpret_cast<const uint4 *>(in + lead);
    auto vector = [&](int64_t v, uint4 raw) {
      Bits *lanes = reinterpret_cast<Bits *>(&raw);
      const int64_t p0 = lead + v * V;
      float xs[V];
      if (sees.all(p0, V)) {
#pragma unroll
        for (int j = 0; j < V; ++j) lanes[j] = D::round(D::to_float(lanes[j]), scale);
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) lanes[j] = value_bits(p0 + j, lanes[j]);
      }
#pragma unroll
      for (int j = 0; j < V; ++j) {
        xs[j] = D::to_float(lanes[j]);
        local_max = fmaxf(local_max, xs[j]);
      }
      if (MODE == kBits) {
        reinterpret_cast<uint4 *>(x_bits + lead)[v] = raw;
      } else {
#pragma unroll
        for (int j = 0; j < V; j += 4)
          *reinterpret_cast<float4 *>(x_float + p0 + j) = make_float4(xs[j], xs[j + 1], xs[j + 2], xs[j + 3]);
      }
    };
    int64_t v = threadIdx.x;
    for (; v + (kBatch - 1) * kLanes < vectors; v += kBatch * kLanes) {
      uint4 raw[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) raw[u] = __ldcs(body + v + u * kLanes);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) vector(v + u * kLanes, raw[u]);
    }
    for (; v < vectors; v += kLanes) vector(v, __ldcs(body + v));
    for (int64_t p = lead + vectors * V + threadIdx.x; p < length; p += kLanes) put(p, value_bits(p, __ldg(in + p)));
  }
  const float maximum = block_max(local_max, scratch);

  auto x_at = [&](int64_t p) -> float {
    if (MODE == kBits) return D::to_float(x_bits[p]);
    if (MODE == kWeights) return x_float[p];
    return D::to_float(value_bits(p, __ldg(in + p)));
  };

  // Pass B: denominator, lane t summing positions t, t + 256, ... in order.
  float sum = 0.0f;
#pragma unroll 4
  for (int64_t p = threadIdx.x; p < length; p += kLanes) {
    const float w = expf(__fsub_rn(x_at(p), maximum));
    if (MODE == kWeights) x_float[p] = w;
    sum = __fadd_rn(sum, w);
  }
  const float denominator = tree_sum(sum, scratch);

  // Pass C: probabilities (optionally stored) and the value projection.
  const Divider divider = make_divider(denominator);
  float projection = 0.0f;
  auto element = [&](int64_t p, float value) {
    const float w = MODE == kWeights ? x_float[p] : expf(__fsub_rn(x_at(p), maximum));
    const float probability = divide(divider, w);
    if (probabilities_out != nullptr) __stcs(probabilities_out + p, probability);
    if (candidates.out != nullptr && candidates.wanted(p)) candidates.put(p, probability);
    projection = __fadd_rn(projection, __fmul_rn(probability, value));
  };
  int64_t p = threadIdx.x;
  for (; p + (kBatch - 1) * kLanes < length; p += kBatch * kLanes) {
    float values[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) values[u] = __ldg(projected_values + p + u * kLanes);
#pragma unroll
    for (int u = 0; u < kBatch; ++u) element(p + u * kLanes, values[u]);
  }
  for (; p < length; p += kLanes) element(p, __ldg(projected_values + p));
  projection = tree_sum(projection, scratch);
  return {maximum, denominator, projection};
}

// Packed float2 IEEE operations (sm_100 add/mul/fma .rn .f32x2), one
// rounding per component.  Written as inline PTX so that the compiler cannot
// merge a product with a following sum into one fused operation (the float2
// builtins allowed that, which changes the rounding of accumulations).
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Pairs of 16-bit logits in one 32-bit word (low half = the earlier element).
template <typename T> struct Packed;
template <> struct Packed<__nv_bfloat16> {
  static constexpr uint32_t kMinusInfinity = 0xff80ff80u;
  static constexpr uint32_t kPlusInfinity = 0x7f807f80u;
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  static __device__ __forceinline__ uint32_t round(float2 v) {  // two RN conversions
    const __nv_bfloat162 r = __floats2bfloat162_rn(v.x, v.y);
    return *reinterpret_cast<const uint32_t *>(&r);
  }
  static __device__ __forceinline__ uint32_t max(uint32_t a, uint32_t b) {  // NaN loses, as in fmaxf
    const __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162 *>(&a),
                                     *reinterpret_cast<const __nv_bfloat162 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
  }
  static __device__ __forceinline__ uint32_t min_nan(uint32_t a, uint32_t b) {  // NaN wins
    const __nv_bfloat162 r = __hmin2_nan(*reinterpret_cast<const __nv_bfloat162 *>(&a),
                                         *reinterpret_cast<const __nv_bfloat162 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
  }
};
template <> struct Packed<__half> {
  static constexpr uint32_t kMinusInfinity = 0xfc00fc00u;
  static constexpr uint32_t kPlusInfinity = 0x7c007c00u;
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&w));
  }
  static __device__ __forceinline__ uint32_t round(float2 v) {
    const __half2 r = __floats2half2_rn(v.x, v.y);
    return *reinterpret_cast<const uint32_t *>(&r);
  }
  static __device__ __forceinline__ uint32_t max(uint32_t a, uint32_t b) {
    const __half2 r = __hmax2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
  }
  static __device__ __forceinline__ uint32_t min_nan(uint32_t a, uint32_t b) {  // NaN wins
    const __half2 r = __hmin2_nan(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
  }
};

// divide() on a pair sharing one denominator: the same residual steps with
// float2 operations (q * (-b) + a is exactly a - q * b before its one rounding).
__device__ __forceinline__ float2 divide2(const Divider &d, float2 a) {
  const float2 y = make_float2(d.y, d.y), minus_b = make_float2(-d.b, -d.b);
  float2 q = mul2_rn(a, y);
  q = fma2_rn(fma2_rn(q, minus_b, a), y, q);
  q = fma2_rn(fma2_rn(q, minus_b, a), y, q);
  const bool fast = d.fast && a.x >= 8.673617379884035e-19f && a.x <= 4294967296.0f &&
                    a.y >= 8.673617379884035e-19f && a.y <= 4294967296.0f;
  if (!fast) q = make_float2(__fdiv_rn(a.x, d.b), __fdiv_rn(a.y, d.b));
  return q;
}

// divide2 without the operand test, for callers that have established it:
// d.fast and both numerators in [2^-60, 2^32].
__device__ __forceinline__ float2 divide2_fast(const Divider &d, float2 a) {
  const float2 y = make_float2(d.y, d.y), minus_b = make_float2(-d.b, -d.b);
  float2 q = mul2_rn(a, y);
  q = fma2_rn(fma2_rn(q, minus_b, a), y, q);
  return fma2_rn(fma2_rn(q, minus_b, a), y, q);
}

// Lowest x - max that keeps expf(x - max) inside divide's fast range:
// expf(-41) = 1.6e-18 > 2^-60 (with room for expf's error), and x <= max
// bounds the weight by 1 from above.
constexpr float kFastExponentFloor = -41.0f;

// Word i of a 16-byte vector (i a compile-time constant after unrolling, so
// the vector stays in registers).
__device__ __forceinline__ uint32_t &word(uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
__device__ __forceinline__ uint32_t word(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Position of lane t's 16-byte chunk within a k-block: XOR-swizzled so that
// both the transposing stores of pass A and the per-lane loads of passes B
// and C touch 8 distinct bank groups per quarter-warp.
__device__ __forceinline__ int chunk_slot(int lane) { return lane ^ ((lane >> 3) & 7); }

// Pass C of the packed stage for one 8-element chunk of one lane (k-block
// kb): x - max, expf, the division, the optional outputs, and the projection
// sum in lane order.  STORE compiles in the store of every probability (the
// drop-in probabilities operator), STASH the candidate stash.  CHECK tests the
// chunk's operands for the fast division; without it the caller has shown
// that every weight of the row is 0 or in [2^-60, 1] (a zero weight divides
// to +0 in the residual form too: every product and residual is +0).
template <typename P, bool STORE, bool STASH, bool CHECK>
__device__ __forceinline__ void packed_chunk(const uint4 chunk, int64_t kb, const float2 minus_max,
                                             const Divider &divider, const float (&current)[8],
                                             float *__restrict__ probabilities_out, const CandidateOut &candidates,
                                             float &projection) {
  // One operand test for the chunk's 8 divisions: its smallest x (NaN if
  // any is NaN) minus max at or above kFastExponentFloor puts every weight
  // in [2^-60, 1] (x - max rounds monotonically in x, and x <= max).
  bool fast = true;
  if constexpr (CHECK) {
    const uint32_t lowest = P::min_nan(P::min_nan(word(chunk, 0), word(chunk, 1)),
                                       P::min_nan(word(chunk, 2), word(chunk, 3)));
    const float2 lowest_d = add2_rn(P::unpack(lowest), minus_max);
    fast = divider.fast && lowest_d.x >= kFastExponentFloor && lowest_d.y >= kFastExponentFloor;
  }
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const float2 d = add2_rn(P::unpack(word(chunk, v)), minus_max);
    const float2 w = make_float2(expf(d.x), expf(d.y));
    const float2 probability = fast ? divide2_fast(divider, w) : make_float2(divide(divider, w.x), divide(divider, w.y));
    if constexpr (STORE) {
      float *out = probabilities_out + threadIdx.x + (kb * 8 + 2 * v) * kLanes;
      __stcs(out, probability.x);
      __stcs(out + kLanes, probability.y);
    }
    if constexpr (STASH) {
      const int64_t p0 = threadIdx.x + (kb * 8 + 2 * v) * kLanes;
      if (candidates.wanted(p0)) candidates.put(p0, probability.x);
      if (candidates.wanted(p0 + kLanes)) candidates.put(p0 + kLanes, probability.y);
    }
    const float2 product = mul2_rn(probability, make_float2(current[2 * v], current[2 * v + 1]));
    projection = __fadd_rn(projection, product.x);
    projection = __fadd_rn(projection, product.y);
  }
}

// row_statistics for MODE == kPacked: 16-bit logits, row 16-byte aligned.
// Stage layout: k-blocks of 8 x 256 elements; lane t's elements t + 256 k,
// k = 8 kb .. 8 kb + 7, sit in order in chunk kb * 256 + chunk_slot(t).  The
// last length % 2048 elements follow in row order.  Pass A reads 8 rows of
// 16-byte vectors per thread (one 8 x 8 tile of lanes x k), rounds and masks
// them in pairs, and transposes the tile with byte permutes; passes B and C
// read one chunk per 8 elements of their lane.  Every element still takes the
// reference's operations in the reference's order.
template <typename T>
__device__ RowResult row_statistics_packed(const T *__restrict__ row, int64_t length, const Visibility sees,
                                           const float *__restrict__ projected_values, float scale,
                                           float *__restrict__ probabilities_out, unsigned char *stage,
                                           float *scratch, const CandidateOut candidates) {
  using P = Packed<T>;
  using D = Dtype<T>;
  constexpr int kBlock = 8 * kLanes;
  const int64_t blocks = length / kBlock;
  const int64_t body = blocks * kBlock;
  uint4 *chunks = reinterpret_cast<uint4 *>(stage);
  unsigned short *tail = reinterpret_cast<unsigned short *>(stage + body * 2);
  const uint4 *in = reinterpret_cast<const uint4 *>(row);
  const float2 scale2 = make_float2(scale, scale);
  const unsigned short neg_inf = minus_infinity<T>();
  uint32_t max_pair = P::kMinusInfinity;
  uint32_t min_pair = P::kPlusInfinity;  // before the mask; NaN wins
  float local_max = -INFINITY;

  // dtype(x * scale), masked, for the 8 elements from p0 (one vector).
  // CHECK tests the mask; without it the caller knows all 8 keys are visible.
  auto prepare = [&](int64_t p0, uint4 raw, auto check) -> uint4 {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      word(raw, i) = P::round(mul2_rn(P::unpack(word(raw, i)), scale2));
      min_pair = P::min_nan(min_pair, word(raw, i));
    }
    if (decltype(check)::value && !sees.all(p0, 8)) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t keep = (sees(p0 + 2 * i) ? 0x0000ffffu : 0u) | (sees(p0 + 2 * i + 1) ? 0xffff0000u : 0u);
        word(raw, i) = (word(raw, i) & keep) | (P::kMinusInfinity & ~keep);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) max_pair = P::max(max_pair, word(raw, i));
    return raw;
  };

  // Pass A, k-blocks: thread item i = (kb, c) covers lanes 8c .. 8c + 7.
  // A row whose k-blocks are all visible (the usual case) skips the mask
  // tests.
  auto k_blocks = [&](auto check) {
  for (int64_t i = threadIdx.x; i < blocks * 32; i += kLanes) {
    const int64_t kb = i >> 5;
    const int c = static_cast<int>(i & 31);
    uint4 raw[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) raw[m] = __ldcs(in + (kb * 8 + m) * 32 + c);
#pragma unroll
    for (int m = 0; m < 8; ++m) raw[m] = prepare((kb * 8 + m) * kLanes + c * 8, raw[m], check);
    uint4 *dst = chunks + kb * kLanes;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t col[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) col[m] = word(raw[m], w);
      const uint4 even = make_uint4(__byte_perm(col[0], col[1], 0x5410), __byte_perm(col[2], col[3], 0x5410),
                                    __byte_perm(col[4], col[5], 0x5410), __byte_perm(col[6], col[7], 0x5410));
      const uint4 odd = make_uint4(__byte_perm(col[0], col[1], 0x7632), __byte_perm(col[2], col[3], 0x7632),
                                   __byte_perm(col[4], col[5], 0x7632), __byte_perm(col[6], col[7], 0x7632));
      dst[chunk_slot(c * 8 + 2 * w)] = even;
      dst[chunk_slot(c * 8 + 2 * w + 1)] = odd;
    }
  }
  };
  if (sees.all(0, body)) k_blocks(std::false_type{});
  else k_blocks(std::true_type{});
  // Pass A, tail: whole vectors, then single elements, in row order.
  const int64_t tail_vectors = (length - body) / 8;
  for (int64_t v = threadIdx.x; v < tail_vectors; v += kLanes)
    reinterpret_cast<uint4 *>(tail)[v] = prepare(body + v * 8, __ldcs(in + body / 8 + v), std::true_type{});
  for (int64_t p = body + tail_vectors * 8 + threadIdx.x; p < length; p += kLanes) {
    const unsigned short raw = reinterpret_cast<const unsigned short *>(row)[p];
    const unsigned short b = sees(p) ? D::round(D::to_float(raw), scale) : neg_inf;
    tail[p - body] = b;
    local_max = fmaxf(local_max, D::to_float(b));
  }
  const float2 pair_max = P::unpack(max_pair);
  local_max = fmaxf(local_max, fmaxf(pair_max.x, pair_max.y));
  // The row's smallest k-block value, negated for the max reduction (+inf
  // when a NaN is present, which turns the row-wide fast division off).
  const float2 pair_min = P::unpack(min_pair);
  const float lowest = fminf(pair_min.x, pair_min.y);
  const float2 extremes =
      block_max2(local_max, isnan(pair_min.x) || isnan(pair_min.y) ? INFINITY : -lowest, scratch);
  const float maximum = extremes.x;

  // Pass B: x - max as x + (-max) (the same IEEE operation), lane order.
  const float2 minus_max = make_float2(-maximum, -maximum);
  const int slot = chunk_slot(threadIdx.x);
  float sum = 0.0f;
  for (int64_t kb = 0; kb < blocks; ++kb) {
    const uint4 chunk = chunks[kb * kLanes + slot];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float2 d = add2_rn(P::unpack(word(chunk, v)), minus_max);
      sum = __fadd_rn(sum, expf(d.x));
      sum = __fadd_rn(sum, expf(d.y));
    }
  }
  for (int64_t p = body + threadIdx.x; p < length; p += kLanes)
    sum = __fadd_rn(sum, expf(__fsub_rn(D::to_float(tail[p - body]), maximum)));
  const float denominator = tree_sum(sum, scratch);

  // Pass C: probabilities and the value projection; the next chunk's
  // projected values are loaded while this chunk computes.  The k-blocks
  // run as up to three loops, each with one compiled chunk body: the
  // candidate columns (the stash) lie in one contiguous range of k-blocks
  // (positions 2048 kb .. 2048 kb + 2047 of every lane; the same answer for
  // the whole CTA), and the loops before and after it carry no stash code.
  const Divider divider = make_divider(denominator);
  const float *values = projected_values + threadIdx.x;
  float projection = 0.0f;
  float next[8];
  if (blocks > 0) {
#pragma unroll
    for (int m = 0; m < 8; ++m) next[m] = __ldg(values + m * kLanes);
  }
  // Row-wide operand test: the smallest k-block x minus max at or above
  // kFastExponentFloor puts every k-block weight in [2^-60, 1], or at 0 for
  // a masked element; then no chunk tests its own.
  const bool row_fast = divider.fast && __fadd_rn(-extremes.y, -maximum) >= kFastExponentFloor;
  auto load_values = [&](int64_t kb, float (&into)[8]) {
#pragma unroll
    for (int m = 0; m < 8; ++m) into[m] = __ldg(values + (kb * 8 + m) * kLanes);
  };
  // Two k-blocks per iteration, their projected values in two buffers, so no
  // buffer is copied; `next` holds the values of k-block kb on entry.
  auto run = [&](int64_t kb_begin, int64_t kb_end, auto store, auto stash, auto check) {
    constexpr bool kStore = decltype(store)::value, kStash = decltype(stash)::value;
    constexpr bool kCheck = decltype(check)::value;
    int64_t kb = kb_begin;
    for (; kb + 1 < kb_end; kb += 2) {
      float second[8];
      load_values(kb + 1, second);
      packed_chunk<P, kStore, kStash, kCheck>(chunks[kb * kLanes + slot], kb, minus_max, divider, next,
                                              probabilities_out, candidates, projection);
      if (kb + 2 < blocks) load_values(kb + 2, next);
      packed_chunk<P, kStore, kStash, kCheck>(chunks[(kb + 1) * kLanes + slot], kb + 1, minus_max, divider,
                                              second, probabilities_out, candidates, projection);
    }
    if (kb < kb_end) {
      float current[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) current[m] = next[m];
      if (kb + 1 < blocks) load_values(kb + 1, next);
      packed_chunk<P, kStore, kStash, kCheck>(chunks[kb * kLanes + slot], kb, minus_max, divider, current,
                                              probabilities_out, candidates, projection);
    }
  };
  using yes = std::true_type;
  using no = std::false_type;
  auto pass_c = [&](auto check) {
    if (probabilities_out != nullptr) {
      run(0, blocks, yes{}, no{}, check);
    } else if (candidates.out != nullptr) {
      const int64_t lo = lmin(blocks, lmax(0, candidates.first / kBlock));
      const int64_t hi = lmin(blocks, lmax(lo, (candidates.last + kBlock - 1) / kBlock));
      run(0, lo, no{}, no{}, check);
      run(lo, hi, no{}, yes{}, check);
      run(hi, blocks, no{}, no{}, check);
    } else {
      run(0, blocks, no{}, no{}, check);
    }
  };
  if (row_fast) pass_c(no{}); else pass_c(yes{});
  for (int64_t p = body + threadIdx.x; p < length; p += kLanes) {
    const float probability = divide(divider, expf(__fsub_rn(D::to_float(tail[p - body]), maximum)));
    if (probabilities_out != nullptr) __stcs(probabilities_out + p, probability);
    if (candidates.out != nullptr && candidates.wanted(p)) candidates.put(p, probability);
    projection = __fadd_rn(projection, __fmul_rn(probability, __ldg(projected_values + p)));
  }
  projection = tree_sum(projection, scratch);
  return {maximum, denominator, projection};
}

}  // namespace rows
}  // namespace lrk
