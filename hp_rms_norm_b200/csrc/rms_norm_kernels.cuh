// Device side of the fused residual-add + RMSNorm family for sm_100a: the
// launch arguments, the per-element arithmetic, and the row kernels.  Only
// rms_norm.cu (launch plans, validation, dispatch, C ABI) includes it.
//
// Per row i (hidden elements, 16-bit storage T, fp32 arithmetic):
//   s_j   = f32(x_ij) + f32(r_ij)
//   r_ij <- round_T(s_j)
//   inv   = rsqrt(eps + sum_j s_j^2 / hidden)          (s_j before rounding)
//   y_ij  = f32(r_ij) * f32(w_j) * inv
//   x_ij <- round_T(y_ij)
// which is the arithmetic of the reference kernel
// (hp_rms_norm/csrc/cuda/hp_rms_norm.cuh:186-207 for the add and the sum of
// squares, :231 for the inverse RMS, :104-110 for the output product).
//
// Beyond the reference's one in-place form, the same kernels compute
//   * plain RMSNorm (no residual: s_j = f32(x_ij), y uses f32(x_ij)),
//   * the result into a separate output tensor (input left unchanged),
//   * an fp8 e4m3 output: e4m3_satfinite(y * (1 / scale)) with a static
//     per-tensor scale, a per-row scale max_j |y_ij| / 448 that is also
//     written out (dynamic per-token quantisation), or one such scale per
//     group of 32/64/128 elements of a row;
//   * an NVFP4 output (e2m1 codes, one e4m3 scale per 16 elements).
//
// The work is purely HBM-bound (8 bytes moved per element, ~6 flops), so the
// kernels are built to keep HBM busy:
//   * every row is read from HBM exactly once and written exactly once: the
//     rounded residual stays in registers between the sum-of-squares pass and
//     the output pass;
//   * all of a thread's loads are issued before any of them is consumed
//     (VPT vectors of input and residual in flight per thread), with 256-bit
//     ld/st.global.v8.b32 where alignment allows;
//   * streamed rows are marked L2 evict_first, the weight row evict_last;
//   * a CTA's first rows are bulk-prefetched into L2 before it waits on the
//     preceding grid (programmatic dependent launch), so their DRAM reads
//     overlap that grid's drain, and each CTA also prefetches the row of the
//     CTA one wave after it; dependents are triggered once the loads are
//     issued in grids of more than one wave (template TL), after the row
//     reduction otherwise (per-plan launch knobs, see default_knobs);
//   * the row is held by part of a warp or one warp (short rows, no shared
//     memory or block barrier at all), one CTA, or a thread-block cluster of
//     up to 8 CTAs
//     whose partial sums meet in distributed shared memory, so that CTAs stay
//     small enough for many to be resident per SM at every hidden size (no
//     occupancy cliff at large hidden);
//   * rows too long for the register-resident kernels use a two-pass kernel,
//     each row split over an eight-CTA cluster, that re-reads its own
//     just-written residual (mostly from L2);
//   * a fifth kernel stages rows in shared memory with TMA bulk copies and
//     mbarriers (plan kind "tma").  Timed against the register-resident
//     kernels at every shape, it is never faster on the fused form, so the
//     launch heuristic never picks it; forced plans reach it.
#pragma once

#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "bulk.cuh"
#include "hp_rms_norm_b200.h"
#include "vec.cuh"

namespace hprn {


// What a launch writes.
enum OutForm : int {
  kOutSame = HPRN_OUT_SAME,                   // 16-bit T into `out` (may be the input)
  kOutFp8Static = HPRN_OUT_FP8_E4M3_STATIC,   // e4m3 with one scale for the tensor
  kOutFp8Dynamic = HPRN_OUT_FP8_E4M3_DYNAMIC,  // e4m3 with one scale per row, written out
  kOutNvfp4 = HPRN_OUT_NVFP4,  // e2m1 pairs + one e4m3 scale per 16 elements (NVFP4)
  kOutFp8Group = HPRN_OUT_FP8_E4M3_GROUP  // e4m3 with one scale per group of a row, written out
};

constexpr float kE4m3Max = 448.0f;
constexpr float kMinAmax = 1e-12f;

struct RmsArgs {
  const uint16_t* x;   // input rows
  const uint16_t* w;   // weight [hidden]
  uint16_t* r;         // residual rows, updated in place (null: plain RMSNorm)
  void* out;           // output rows (T or e4m3 bytes)
  const float* scale;  // static fp8 scale, or the NVFP4 global scale (one float)
  float* row_scales;   // dynamic fp8 scales, one per row
  uint8_t* block_scales;  // NVFP4 block scales, rows x hidden/16 e4m3 bytes
  int64_t rows;
  int64_t x_stride;    // elements between rows
  int64_t r_stride;
  int64_t out_stride;
  int32_t nvec;        // vectors per row (hidden / elements-per-vector)
  int32_t slice_vecs;  // vectors per CTA when a cluster splits the row
  int32_t rows_per_cta;
  float eps;
  float inv_hidden;
  // Per-group fp8 scales (in row_scales): the scale of row i, group g sits
  // at i * gs_row + g * gs_group; a group is group_vecs vectors.
  int64_t gs_row;
  int64_t gs_group;
  int32_t group_vecs;
  int32_t scale_pow2;  // round group scales up to powers of two
  int32_t lanes_per_row;  // warp kind: lanes holding one row (1..32, a power of two)
  // TMA-staged kernel only: the limit of each per-row mbarrier wait, and a
  // row (of this call, -1: none) whose staged copy is made to expect
  // kStallBytes more than it delivers, so that its wait runs out (a test hook:
  // hprn_test_stall_bulk_copy).
  int64_t stall_row;
  uint64_t wait_limit_ns;
  // CTAs blockIdx.x < prefetch_ctas prefetch their first rows into L2 before
  // the programmatic-launch wait (0: none; the grid's first wave; or all).
  int64_t prefetch_ctas;
  // > 0: after issuing its own loads, each CTA also prefetches its slice of
  // the row this many rows ahead, the row of the CTA that will take its place
  // one wave later.
  int64_t prefetch_ahead_rows;
  // Where a CTA triggers its dependents (pdl_trigger): 0 after its last
  // store, 1 after the row reduction.  Triggering once the loads (and
  // prefetches) are issued is a separate kernel instance (template TL), not
  // this runtime value: with the trigger compiled in that early, even
  // untaken, short single-wave launches ran up to 15% slower.  Instances
  // without TL treat 2 as 1.
  int32_t early_trigger;
};

// Prefetches into L2 the vectors [v_begin, v_end) of the row
// a.prefetch_ahead_rows after `row` (input, and residual with RES), when that
// row is part of this launch.  One thread per row slice calls it, after its
// CTA's own loads are issued: the DRAM reads of the row a CTA of the next wave
// will load then overlap this CTA's reduction and epilogue, without registers.
template <int VEC, bool RES>
__device__ __forceinline__ void prefetch_row_ahead(const RmsArgs& a, int64_t row, int v_begin,
                                                   int v_end) {
  const int64_t ahead = row + a.prefetch_ahead_rows;
  if (a.prefetch_ahead_rows > 0 && ahead < a.rows && v_end > v_begin) {
    const int64_t first = static_cast<int64_t>(v_begin) * Vec<VEC>::kElems;
    const uint64_t bytes = static_cast<uint64_t>(v_end - v_begin) * VEC;
    prefetch_l2(a.x + ahead * a.x_stride + first, bytes);
    if constexpr (RES) prefetch_l2(a.r + ahead * a.r_stride + first, bytes);
  }
}

// Element pairs go through Blackwell's packed fp32 instructions
// (__fadd2_rn / __fmul2_rn / __ffma2_rn: add/mul/fma.rn.f32x2), and squares
// and products of two 16-bit operands through its mixed-precision
// fma.rn.f32.{bf16,f16} (fma_pair / mul_pair), which reads the 16-bit halves
// directly instead of unpacking them.  Each rounds exactly as the scalar fp32
// instruction does (nearest even, no flush to zero), so the results are those
// of scalar code, bit for bit, in fewer instructions.

// Adds residual into input in fp32, keeps the rounded sum in `xv`, and
// accumulates the squares of the unrounded sums (even elements into a0, odd
// into a1).
template <typename T, int VEC>
__device__ __forceinline__ void add_round(Vec<VEC>& xv, const Vec<VEC>& rv, float& a0, float& a1) {
  if constexpr (VEC == 2) {
    const float s = unpack1<T>(xv.h) + unpack1<T>(rv.h);
    a0 = fmaf(s, s, a0);
    xv.h = pack1<T>(s);
  } else {
    float2 acc = make_float2(a0, a1);
#pragma unroll
    for (int k = 0; k < Vec<VEC>::kWords; ++k) {
      const float2 s = __fadd2_rn(unpack2<T>(xv.w[k]), unpack2<T>(rv.w[k]));
      acc = __ffma2_rn(s, s, acc);
      xv.w[k] = pack2<T>(s.x, s.y);
    }
    a0 = acc.x;
    a1 = acc.y;
  }
}

// Sum of squares of the input alone (plain RMSNorm).
template <typename T, int VEC>
__device__ __forceinline__ void square_sum(const Vec<VEC>& xv, float& a0, float& a1) {
  if constexpr (VEC == 2) {
    const float s = unpack1<T>(xv.h);
    a0 = fmaf(s, s, a0);
  } else {
    float2 acc = make_float2(a0, a1);
#pragma unroll
    for (int k = 0; k < Vec<VEC>::kWords; ++k) acc = fma_pair<T>(xv.w[k], xv.w[k], acc);
    a0 = acc.x;
    a1 = acc.y;
  }
}

// round_T((f32(r) * f32(w)) * inv), multiplied in the reference's order.
template <typename T, int VEC>
__device__ __forceinline__ Vec<VEC> normalize(const Vec<VEC>& rv, const Vec<VEC>& wv, float inv) {
  Vec<VEC> o;
  if constexpr (VEC == 2) {
    o.h = pack1<T>(unpack1<T>(rv.h) * unpack1<T>(wv.h) * inv);
  } else {
    const float2 inv2 = make_float2(inv, inv);
#pragma unroll
    for (int k = 0; k < Vec<VEC>::kWords; ++k) {
      const float2 y = __fmul2_rn(mul_pair<T>(rv.w[k], wv.w[k]), inv2);
      o.w[k] = pack2<T>(y.x, y.y);
    }
  }
  return o;
}

// f32(r_j) * f32(w_j) for the elements of one vector, as pairs: the common
// factor of every quantised output.  Computed once per element and shared by
// the amax and the quantiser.
template <int VEC>
struct Prod {
  float2 p[Vec<VEC>::kWords];
};

template <typename T, int VEC>
__device__ __forceinline__ Prod<VEC> product(const Vec<VEC>& rv, const Vec<VEC>& wv) {
  Prod<VEC> o;
#pragma unroll
  for (int k = 0; k < Vec<VEC>::kWords; ++k) o.p[k] = mul_pair<T>(rv.w[k], wv.w[k]);
  return o;
}

// max(m, |a|, |b|) in one sm_100 three-input max.f32.  NaN operands are
// ignored, as by fmaxf; no flush to zero.
__device__ __forceinline__ float max_abs2(float m, float a, float b) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return d;
}

// max_j |p_j| over one vector of products, folded into m.  The amax of
// y_j = p_j * inv is this times inv, rounded once: inv > 0 and
// round-to-nearest is monotone, so max_j |RN(p_j * inv)| = RN(max_j |p_j| * inv)
// exactly, with one multiply per row (or group) instead of one per element.
template <int VEC>
__device__ __forceinline__ float prod_amax(const Prod<VEC>& p, float m) {
#pragma unroll
  for (int k = 0; k < Vec<VEC>::kWords; ++k) m = max_abs2(m, p.p[k].x, p.p[k].y);
  return m;
}

// e4m3_satfinite((p * inv) * inv_scale) for one vector of products: VEC/2
// output bytes, element order preserved.
template <int VEC>
__device__ __forceinline__ Vec<VEC / 2> quantize_e4m3(const Prod<VEC>& p, float inv,
                                                      float inv_scale) {
  static_assert(VEC >= 8, "fp8 output needs at least 4 elements per vector");
  Vec<VEC / 2> o;
  const float2 inv2 = make_float2(inv, inv);
  const float2 is2 = make_float2(inv_scale, inv_scale);
#pragma unroll
  for (int k = 0; k < Vec<VEC>::kWords; k += 2) {
    uint32_t word = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 q = __fmul2_rn(__fmul2_rn(p.p[k + h], inv2), is2);
      const __nv_fp8x2_storage_t b = __nv_cvt_float2_to_fp8x2(q, __NV_SATFINITE, __NV_E4M3);
      word |= static_cast<uint32_t>(b) << (16 * h);
    }
    o.w[k / 2] = word;
  }
  return o;
}

// NVFP4 for one 32-byte vector (exactly one 16-element block):
//   sf = e4m3_satfinite(gs * (max_j |y_j| / 6)),  q_j = e2m1(y_j * (gs / sf))
// (q = 0 when sf is 0).  Returns the 8 packed bytes (element 2k in the low
// nibble of byte k) and the scale byte.
template <typename T>
__device__ __forceinline__ Vec<8> quantize_nvfp4(const Vec<32>& rv, const Vec<32>& wv, float inv,
                                                 float gs, uint8_t* sf_out) {
  float2 y[8];
  const float2 inv2 = make_float2(inv, inv);
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    y[k] = __fmul2_rn(mul_pair<T>(rv.w[k], wv.w[k]), inv2);
    amax = max_abs2(amax, y[k].x, y[k].y);
  }
  const __nv_fp8_storage_t sf = __nv_cvt_float_to_fp8(gs * (amax / 6.0f), __NV_SATFINITE, __NV_E4M3);
  const float sfv = __half2float(__half(__nv_cvt_fp8_to_halfraw(sf, __NV_E4M3)));
  const float qs = sfv != 0.f ? gs / sfv : 0.f;
  const float2 qs2 = make_float2(qs, qs);
  Vec<8> o;
#pragma unroll
  for (int w = 0; w < 2; ++w)
    o.w[w] = e2m1x8(__fmul2_rn(y[4 * w], qs2), __fmul2_rn(y[4 * w + 1], qs2),
                    __fmul2_rn(y[4 * w + 2], qs2), __fmul2_rn(y[4 * w + 3], qs2));
  *sf_out = sf;
  return o;
}

// Butterfly reductions: every lane ends with the same bits.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Butterflies over aligned groups of `width` lanes (a power of two, 1..32):
// every lane ends with its group's result; width 32 is warp_sum / warp_max.
__device__ __forceinline__ float lane_group_sum(float v, int width) {
  for (int o = width >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float lane_group_max(float v, int width) {
  for (int o = width >> 1; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Stores `v` into the shared-memory word at `local` in CTA `rank` of this cluster.
__device__ __forceinline__ void st_cluster_f32(float* local, uint32_t rank, float v) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local));
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

// Inverse of the static fp8 scale, or the NVFP4 global scale itself, read
// after the programmatic-launch wait.
template <int OUT>
__device__ __forceinline__ float static_inv_scale(const RmsArgs& a) {
  if constexpr (OUT == kOutFp8Static) return 1.0f / __ldg(a.scale);
  if constexpr (OUT == kOutNvfp4) return __ldg(a.scale);
  return 1.0f;
}

// Writes the e4m3 codes of one output vector from its products.
template <int VEC>
__device__ __forceinline__ void store_e4m3(const RmsArgs& a, int64_t row, int64_t v,
                                           const Prod<VEC>& p, float inv, float inv_scale) {
  uint8_t* o = static_cast<uint8_t*>(a.out) + row * a.out_stride + v * Vec<VEC>::kElems;
  st_global<VEC / 2>(o, quantize_e4m3<VEC>(p, inv, inv_scale));
}

// Writes one output vector of row `row` at vector index v.
template <typename T, int VEC, int OUT>
__device__ __forceinline__ void store_out(const RmsArgs& a, int64_t row, int64_t v,
                                          const Vec<VEC>& rv, const Vec<VEC>& wv, float inv,
                                          float inv_scale) {
  constexpr int EPV = Vec<VEC>::kElems;
  if constexpr (OUT == kOutSame) {
    uint16_t* o = static_cast<uint16_t*>(a.out) + row * a.out_stride + v * EPV;
    st_global<VEC>(o, normalize<T, VEC>(rv, wv, inv));
  } else if constexpr (OUT == kOutNvfp4) {
    static_assert(VEC == 32, "NVFP4 blocks are one 32-byte vector of 16 elements");
    uint8_t sf;
    // out_stride counts fp4 elements: byte offset = elements / 2.
    uint8_t* o = static_cast<uint8_t*>(a.out) + (row * a.out_stride + v * EPV) / 2;
    st_global<8>(o, quantize_nvfp4<T>(rv, wv, inv, inv_scale, &sf));
    a.block_scales[row * a.nvec + v] = sf;
  } else {
    store_e4m3<VEC>(a, row, v, product<T, VEC>(rv, wv), inv, inv_scale);
  }
}

// The weight vector for output vector v.  With a residual, the weight was
// loaded before the reduction (its latency hides behind the barrier) and is
// passed in; without one, it is loaded here, at use: a plain row holds half
// the bytes per thread, so keeping the weight out of the registers live
// across the barrier lets more CTAs reside per SM (at hidden 24576, two
// 768-thread CTAs instead of one), which is what a plain row's bandwidth
// depends on.
template <int VEC, bool RES>
__device__ __forceinline__ Vec<VEC> weight_vec(const RmsArgs& a, int64_t v, const Vec<VEC>& held,
                                               uint64_t pol_keep) {
  if constexpr (RES) return held;
  return ld_weight<VEC>(a.w + v * Vec<VEC>::kElems, pol_keep);
}

// The smallest power of two >= s, for a positive normal float s (exact: the
// exponent field goes up by one unless the mantissa field is zero).
__device__ __forceinline__ float pow2_ceil(float s) {
  uint32_t u = __float_as_uint(s);
  if (u & 0x7fffffu) u = (u & 0xff800000u) + 0x800000u;
  return __uint_as_float(u);
}

// Per-token-group fp8 for output vector v (in: v is inside the row slice).
// The vectors of one group sit in group_vecs consecutive lanes of a warp
// (vector index = a group-aligned base + lane), so the group amax is a
// butterfly over log2(group_vecs) lanes: every lane of the warp must call
// this, lanes outside the slice with in = false.  max |y| over a vector is
// max |r * w| times inv, rounded once (exact, see prod_amax); the products
// are formed once for the amax and the quantiser.
template <typename T, int VEC, bool RES>
__device__ __forceinline__ void store_group_fp8(const RmsArgs& a, int64_t row, int v, bool in,
                                                const Vec<VEC>& rv, const Vec<VEC>& held,
                                                float inv, uint64_t pol_keep) {
  Vec<VEC> wv = held;
  if (!RES && in) wv = weight_vec<VEC, RES>(a, v, held, pol_keep);
  const Prod<VEC> p = product<T, VEC>(rv, wv);
  float m = in ? prod_amax<VEC>(p, 0.f) * inv : 0.f;
  // group_vecs is 2, 4 or 8 (groups of 32/64/128 elements, 16 per vector).
#pragma unroll
  for (int o = 1; o < 8; o <<= 1)
    if (o < a.group_vecs) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float scale = fmaxf(m, kMinAmax) / kE4m3Max;
  if (a.scale_pow2) scale = pow2_ceil(scale);
  if (in) {
    store_e4m3<VEC>(a, row, v, p, inv, 1.0f / scale);
    if ((v & (a.group_vecs - 1)) == 0) {  // the group's first vector; v >= 0
      const int g = v >> (__ffs(a.group_vecs) - 1);
      a.row_scales[row * a.gs_row + static_cast<int64_t>(g) * a.gs_group] = scale;
    }
  }
}

// Whether a dynamic-fp8 kernel keeps the fp32 products r * w (16 registers
// per 32-byte vector) live across the row reduction, so that the output pass
// only scales, converts and stores, instead of keeping the 16-bit row (8
// registers) and forming the products a second time.  A fused row holds r
// and w across the reduction anyway, so its products cost no extra
// registers.  A plain row holds only x: at up to two vectors per thread the
// products fit beside it (4096 x 8192: 19.0 vs 20.9 us), at four they cost
// half the resident CTAs (4096 x 32768: 89 vs 72 us).
__host__ __device__ constexpr bool hold_products(bool res, int vpt) { return res || vpt <= 2; }

// ---------------------------------------------------------------------------
// Kernel 1: rows of at most 4 * 32 vectors, each held by `lanes_per_row`
// lanes of one warp (a whole warp, or 32 / lanes_per_row rows per warp for
// short rows: 1-32 lanes, a power of two), reduced by a butterfly over those
// lanes.  No shared memory, no block barrier.  Lanes past the last row stay
// in the warp (their loads and stores are skipped) so every shuffle has all
// 32 lanes.
template <typename T, int VEC, int VPT, bool RES, int OUT, bool TL>
__global__ void __launch_bounds__(256) rms_norm_warp_rows(RmsArgs a) {
  constexpr int EPV = Vec<VEC>::kElems;
  const int lpr = a.lanes_per_row;
  const int sub = threadIdx.x & (lpr - 1);
  const int64_t row = static_cast<int64_t>(blockIdx.x) * a.rows_per_cta + threadIdx.x / lpr;
  const bool active = row < a.rows;
  const uint16_t* xr = a.x + row * a.x_stride;
  uint16_t* rr = RES ? a.r + row * a.r_stride : nullptr;
  if (active && sub == 0 && blockIdx.x < a.prefetch_ctas) {
    prefetch_l2(xr, static_cast<uint64_t>(a.nvec) * VEC);
    if constexpr (RES) prefetch_l2(rr, static_cast<uint64_t>(a.nvec) * VEC);
  }
  pdl_wait();
  const uint64_t pol_stream = policy_evict_first();
  const uint64_t pol_keep = policy_evict_last();

  Vec<VEC> xv[VPT], rv[VPT], wv[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = sub + lpr * j;
    if (active && v < a.nvec) {
      xv[j] = ld_stream<VEC>(xr + v * EPV, pol_stream);
      if constexpr (RES) rv[j] = ld_stream<VEC>(rr + v * EPV, pol_stream);
    }
  }
  if (active && sub == 0) prefetch_row_ahead<VEC, RES>(a, row, 0, a.nvec);
  if constexpr (TL) pdl_trigger();
  float a0 = 0.f, a1 = 0.f;
  // Dynamic fp8: max |r * w| does not depend on inv, so it is reduced next to
  // the sum of squares and scaled by inv once (see prod_amax).  The products
  // r * w are held across the reduction for the output pass (kHold, see
  // hold_products).
  constexpr bool kAmax = OUT == kOutFp8Dynamic;
  constexpr bool kHold = kAmax && hold_products(RES, VPT);
  Prod<kHold ? VEC : 8> pv[VPT];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = sub + lpr * j;
    if (active && v < a.nvec) {
      if constexpr (RES) {
        add_round<T, VEC>(xv[j], rv[j], a0, a1);
        st_global<VEC>(rr + v * EPV, xv[j]);
        wv[j] = ld_weight<VEC>(a.w + v * EPV, pol_keep);
      } else {
        square_sum<T, VEC>(xv[j], a0, a1);
        if constexpr (kAmax) {
          const Prod<VEC> p = product<T, VEC>(xv[j], weight_vec<VEC, RES>(a, v, wv[j], pol_keep));
          m = prod_amax<VEC>(p, m);
          if constexpr (kHold) pv[j] = p;
        }
      }
    }
  }
  if constexpr (RES && kAmax) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = sub + lpr * j;
      if (active && v < a.nvec) {
        pv[j] = product<T, VEC>(xv[j], wv[j]);
        m = prod_amax<VEC>(pv[j], m);
      }
    }
  }
  float inv_scale = static_inv_scale<OUT>(a);
  const float inv = rsqrtf(fmaf(lane_group_sum(a0 + a1, lpr), a.inv_hidden, a.eps));
  if (!TL && a.early_trigger >= 1) pdl_trigger();
  if constexpr (OUT == kOutFp8Dynamic) {
    const float scale = fmaxf(lane_group_max(m, lpr) * inv, kMinAmax) / kE4m3Max;
    inv_scale = 1.0f / scale;
    if (sub == 0 && active) a.row_scales[row] = scale;
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = sub + lpr * j;
    if constexpr (OUT == kOutFp8Group) {
      store_group_fp8<T, VEC, RES>(a, row, v, active && v < a.nvec, xv[j], wv[j], inv, pol_keep);
    } else if constexpr (kHold) {
      if (active && v < a.nvec) store_e4m3<VEC>(a, row, v, pv[j], inv, inv_scale);
    } else if (active && v < a.nvec) {
      store_out<T, VEC, OUT>(a, row, v, xv[j], weight_vec<VEC, RES>(a, v, wv[j], pol_keep), inv,
                             inv_scale);
    }
  }
  if (!TL && a.early_trigger == 0) pdl_trigger();
}

// Largest CTA a cta/cluster kernel with VPT vectors per thread is compiled
// for: the register budget per thread (65536 / max threads) must hold the
// 3 * VPT vectors in flight without spilling.
__host__ __device__ constexpr int cta_max_threads(int vpt) {
  return vpt <= 2 ? 1024 : (vpt <= 4 ? 512 : 256);
}

// CTAs of cta_max_threads(VPT) threads each SM must hold at once (0: no
// minimum, the compiler's own register choice).  A plain
// 16-bit row at two vectors per thread (one CTA per row) runs in 1024-thread
// CTAs at hidden 32768 and needs two of them per SM, i.e. at most 32
// registers per thread (with 33 it ran at 0.83 of the copy peak, not 1.01).
__host__ __device__ constexpr int cta_min_blocks(int vpt, bool cluster, bool res, int out) {
  return (vpt == 2 && !cluster && !res && out == kOutSame) ? 2 : 0;
}

// ---------------------------------------------------------------------------
// Kernel 2: one CTA per row slice; with CLUSTER, the row is split over the
// CTAs of a thread-block cluster (launched with cluster dims (n, 1, 1)) and
// the per-CTA partials (sum of squares, and for dynamic fp8 the amax) are
// pushed into every peer's shared memory, so each CTA finishes each reduction
// locally after one cluster barrier and no CTA touches a peer's memory
// afterwards.
// Whether a CTA kernel instance has the launch knobs (L2 prefetch before the
// dependency wait, trigger after the reduction).  The plain NVFP4 and
// per-group fp8 forms at four vectors per thread are issue-bound, and with
// the knobs' code compiled in they ran 1.5-2% slower at hidden 16384-32768
// even with both knobs off (plain NVFP4 at 4096 x 32768: 60.6 against 59.5
// us); they keep their trigger at the end and no prefetch.
__host__ __device__ constexpr bool cta_has_knobs(bool res, int out, int vpt) {
  return res || (out != kOutNvfp4 && out != kOutFp8Group) || vpt < 4;
}

template <typename T, int VEC, int VPT, bool CLUSTER, bool RES, int OUT, bool TL>
__global__ void __launch_bounds__(cta_max_threads(VPT), cta_min_blocks(VPT, CLUSTER, RES, OUT))
    rms_norm_cta_rows(RmsArgs a) {
  constexpr bool kKnobs = cta_has_knobs(RES, OUT, VPT);
  static_assert(kKnobs || !TL, "the knob-less instances trigger at their end only");
  constexpr int EPV = Vec<VEC>::kElems;
  __shared__ float warp_part[32];
  __shared__ float warp_amax[32];
  __shared__ float cta_part[8];
  __shared__ float cta_amax[8];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int nwarps = nthreads >> 5;

  int64_t row;
  int v_begin = 0, v_end = a.nvec;
  uint32_t crank = 0, csize = 1;
  if constexpr (CLUSTER) {
    crank = cluster_ctarank();
    csize = cluster_nctarank();
    row = cluster_id_x();
    v_begin = static_cast<int>(crank) * a.slice_vecs;
    v_end = min(v_begin + a.slice_vecs, a.nvec);
  } else {
    row = blockIdx.x;
  }
  const uint16_t* xr = a.x + row * a.x_stride;
  uint16_t* rr = RES ? a.r + row * a.r_stride : nullptr;
  if (kKnobs && tid == 0 && v_end > v_begin && blockIdx.x < a.prefetch_ctas) {
    const uint64_t bytes = static_cast<uint64_t>(v_end - v_begin) * VEC;
    prefetch_l2(xr + static_cast<int64_t>(v_begin) * EPV, bytes);
    if constexpr (RES) prefetch_l2(rr + static_cast<int64_t>(v_begin) * EPV, bytes);
  }
  pdl_wait();
  // Phase 1 of the cluster barrier: completes once every CTA of the cluster
  // is running, which makes their shared memory safe to write.
  if constexpr (CLUSTER) cluster_arrive_relaxed();
  const uint64_t pol_stream = policy_evict_first();
  const uint64_t pol_keep = policy_evict_last();

  Vec<VEC> xv[VPT], rv[VPT], wv[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = v_begin + tid + j * nthreads;
    if (v < v_end) {
      xv[j] = ld_stream<VEC>(xr + static_cast<int64_t>(v) * EPV, pol_stream);
      if constexpr (RES) rv[j] = ld_stream<VEC>(rr + static_cast<int64_t>(v) * EPV, pol_stream);
    }
  }
  if (kKnobs && tid == 0) prefetch_row_ahead<VEC, RES>(a, row, v_begin, v_end);
  if constexpr (TL) pdl_trigger();
  // Dynamic fp8: max |r * w| does not depend on inv, so it travels with the
  // sum of squares through the same barrier (and cluster phase) and is scaled
  // by inv once at the end (see prod_amax).  The products r * w are held
  // across the reduction for the output pass (kHold, see hold_products).
  constexpr bool kAmax = OUT == kOutFp8Dynamic;
  constexpr bool kHold = kAmax && hold_products(RES, VPT);
  Prod<kHold ? VEC : 8> pv[VPT];
  float a0 = 0.f, a1 = 0.f;
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = v_begin + tid + j * nthreads;
    if (v < v_end) {
      if constexpr (RES) {
        add_round<T, VEC>(xv[j], rv[j], a0, a1);
        st_global<VEC>(rr + static_cast<int64_t>(v) * EPV, xv[j]);
        wv[j] = ld_weight<VEC>(a.w + static_cast<int64_t>(v) * EPV, pol_keep);
      } else {
        square_sum<T, VEC>(xv[j], a0, a1);
        if constexpr (kAmax) {
          const Prod<VEC> p = product<T, VEC>(xv[j], weight_vec<VEC, RES>(a, v, wv[j], pol_keep));
          m = prod_amax<VEC>(p, m);
          if constexpr (kHold) pv[j] = p;
        }
      }
    }
  }
  if constexpr (RES && kAmax) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = v_begin + tid + j * nthreads;
      if (v < v_end) {
        pv[j] = product<T, VEC>(xv[j], wv[j]);
        m = prod_amax<VEC>(pv[j], m);
      }
    }
  }
  float inv_scale = static_inv_scale<OUT>(a);  // read before the barrier hides its latency
  const float wsum = warp_sum(a0 + a1);
  if constexpr (kAmax) m = warp_max(m);
  if (lane == 0) {
    warp_part[warp] = wsum;
    if constexpr (kAmax) warp_amax[warp] = m;
  }
  __syncthreads();
  float total = warp_sum(lane < nwarps ? warp_part[lane] : 0.f);
  float amax = kAmax ? warp_max(lane < nwarps ? warp_amax[lane] : 0.f) : 0.f;
  if constexpr (CLUSTER) {
    cluster_wait();  // phase 1: all peers are running
    if (warp == 0 && lane < static_cast<int>(csize)) {
      st_cluster_f32(&cta_part[crank], lane, total);
      if constexpr (kAmax) st_cluster_f32(&cta_amax[crank], lane, amax);
    }
    cluster_arrive_release();
    cluster_wait();  // phase 2: every CTA's partials have landed in every CTA
    total = warp_sum(lane < static_cast<int>(csize) ? cta_part[lane] : 0.f);
    if constexpr (kAmax) amax = warp_max(lane < static_cast<int>(csize) ? cta_amax[lane] : 0.f);
  }
  const float inv = rsqrtf(fmaf(total, a.inv_hidden, a.eps));
  if (kKnobs && !TL && a.early_trigger >= 1) pdl_trigger();
  if constexpr (kAmax) {
    const float scale = fmaxf(amax * inv, kMinAmax) / kE4m3Max;
    inv_scale = 1.0f / scale;
    if (crank == 0 && tid == 0) a.row_scales[row] = scale;
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = v_begin + tid + j * nthreads;
    if constexpr (OUT == kOutFp8Group) {
      store_group_fp8<T, VEC, RES>(a, row, v, v < v_end, xv[j], wv[j], inv, pol_keep);
    } else if constexpr (kHold) {
      if (v < v_end) store_e4m3<VEC>(a, row, v, pv[j], inv, inv_scale);
    } else if (v < v_end) {
      store_out<T, VEC, OUT>(a, row, v, xv[j], weight_vec<VEC, RES>(a, v, wv[j], pol_keep), inv,
                             inv_scale);
    }
  }
  if (!kKnobs || (!TL && a.early_trigger == 0)) pdl_trigger();
}

// ---------------------------------------------------------------------------
// Kernel 3: rows longer than the register-resident kernels hold (16-bit
// output only).  Pass 1 streams the input (and residual) from HBM, writes the
// rounded residual and sums squares; pass 2 re-reads each thread's own
// residual (or input) vectors from L2 (.cg), multiplies by the weight and
// writes the output.  What pass 2 reads is written (fused) or read (plain) in
// pass 1 with an L2 evict_last policy, and read back with evict_first: the
// streamed rows (evict_first) then do not push it out of L2 before its second
// use, so at 64 x 1M the launch reads 1.03x its algorithmic bytes from DRAM
// instead of 1.17x.  With CLUSTER, the row is split over the CTAs of a
// thread-block cluster (for row counts too small to fill the SMs one CTA per
// row); each CTA pushes its partial sum into every peer's shared memory, and
// one cluster barrier completes the row's sum between the passes.
constexpr int kTwoPassThreads = 512;
// Vectors each thread has in flight per chunk of a two-pass row.
constexpr int kTwoPassUnroll = 4;

template <typename T, int VEC, bool RES, bool CLUSTER>
__global__ void __launch_bounds__(kTwoPassThreads) rms_norm_two_pass(RmsArgs a) {
  constexpr int EPV = Vec<VEC>::kElems;
  constexpr int U = kTwoPassUnroll;
  __shared__ float warp_part[32];
  __shared__ float cta_part[8];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nthreads = blockDim.x;
  int64_t row;
  int v_begin = 0, v_end = a.nvec;
  uint32_t crank = 0, csize = 1;
  if constexpr (CLUSTER) {
    crank = cluster_ctarank();
    csize = cluster_nctarank();
    row = cluster_id_x();
    v_begin = static_cast<int>(crank) * a.slice_vecs;
    v_end = min(v_begin + a.slice_vecs, a.nvec);
  } else {
    row = blockIdx.x;
  }
  const uint16_t* xr = a.x + row * a.x_stride;
  uint16_t* rr = RES ? a.r + row * a.r_stride : nullptr;
  uint16_t* orow = static_cast<uint16_t*>(a.out) + row * a.out_stride;
  if (tid == 0 && v_end > v_begin && blockIdx.x < a.prefetch_ctas) {  // pass 1's first chunk
    const uint64_t bytes = static_cast<uint64_t>(min(U * nthreads, v_end - v_begin)) * VEC;
    prefetch_l2(xr + static_cast<int64_t>(v_begin) * EPV, bytes);
    if constexpr (RES) prefetch_l2(rr + static_cast<int64_t>(v_begin) * EPV, bytes);
  }
  pdl_wait();
  if constexpr (CLUSTER) cluster_arrive_relaxed();  // phase 1: completes once every peer is running
  if (tid == 0) prefetch_row_ahead<VEC, RES>(a, row, v_begin, min(v_begin + U * nthreads, v_end));
  const uint64_t pol_stream = policy_evict_first();
  const uint64_t pol_keep = policy_evict_last();

  float a0 = 0.f, a1 = 0.f;
  for (int base = v_begin; base < v_end; base += U * nthreads) {
    Vec<VEC> xv[U], rv[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int v = base + tid + j * nthreads;
      if (v < v_end) {
        // The plain form reads its input again in pass 2: keep it in L2.
        xv[j] = ld_stream<VEC>(xr + static_cast<int64_t>(v) * EPV, RES ? pol_stream : pol_keep);
        if constexpr (RES) rv[j] = ld_stream<VEC>(rr + static_cast<int64_t>(v) * EPV, pol_stream);
      }
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int v = base + tid + j * nthreads;
      if (v < v_end) {
        if constexpr (RES) {
          add_round<T, VEC>(xv[j], rv[j], a0, a1);
          st_global_hint<VEC>(rr + static_cast<int64_t>(v) * EPV, xv[j], pol_keep);
        } else {
          square_sum<T, VEC>(xv[j], a0, a1);
        }
      }
    }
  }
  const float wsum = warp_sum(a0 + a1);
  if (lane == 0) warp_part[warp] = wsum;
  __syncthreads();
  float total = warp_sum(lane < (nthreads >> 5) ? warp_part[lane] : 0.f);
  if constexpr (CLUSTER) {
    cluster_wait();  // phase 1: all peers are running
    if (warp == 0 && lane < static_cast<int>(csize)) st_cluster_f32(&cta_part[crank], lane, total);
    cluster_arrive_release();
    cluster_wait();  // phase 2: every CTA's partial has landed in every CTA
    total = warp_sum(lane < static_cast<int>(csize) ? cta_part[lane] : 0.f);
  }
  const float inv = rsqrtf(fmaf(total, a.inv_hidden, a.eps));
  if (a.early_trigger) pdl_trigger();

  // Pass 2 reads the values this thread wrote (residual) or read (input) in pass 1.
  const uint16_t* src = RES ? rr : xr;
  for (int base = v_begin; base < v_end; base += U * nthreads) {
    Vec<VEC> sv[U], wv[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int v = base + tid + j * nthreads;
      if (v < v_end) {
        sv[j] = ld_l2_hint<VEC>(src + static_cast<int64_t>(v) * EPV, pol_stream);
        wv[j] = ld_weight<VEC>(a.w + static_cast<int64_t>(v) * EPV, pol_keep);
      }
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int v = base + tid + j * nthreads;
      if (v < v_end) {
        st_global<VEC>(orow + static_cast<int64_t>(v) * EPV, normalize<T, VEC>(sv[j], wv[j], inv));
      }
    }
  }
  if (!a.early_trigger) pdl_trigger();
}

// ---------------------------------------------------------------------------
// Kernel 4: rows staged in shared memory by TMA bulk copies (16-bit output).
// A persistent grid (as many CTAs as fit on the SMs) walks rows blockIdx.x,
// + gridDim.x, ...; one thread issues, per row, a 1-D cp.async.bulk of the
// input row (and one of the residual row) into a ring of `stages` row buffers,
// each completing on its own mbarrier, so a CTA keeps `stages` rows in flight
// with two instructions per row whatever the row length.  All threads wait on
// the stage's mbarrier, take their 16- or 32-byte vectors from shared memory and
// finish the row as the register kernels do.  The reduction barrier doubles as
// the stage's release: right after it the issuing thread refills the stage
// with the row `stages` ahead.  The weight stays in registers for every row.
// A wait that gives up (a copy that never completed) ends the CTA after the
// copies it still has in flight have landed, and counts in g_wait_timeouts.
// The residual and the output of a row are stored only after every thread's
// wait for it succeeded, so a CTA that gives up leaves the row it gave up on,
// and every later row of its share, untouched (input and residual as they
// were); rows it finished before are complete.
constexpr int kTmaMaxStages = 16;
// Bytes a stalled row's phase expects beyond its copies (test hook).
constexpr uint32_t kStallBytes = 16;
// Shared memory per CTA kept out of the dynamic ring: the mbarriers and the
// reduction partials (384 bytes), rounded up.
constexpr int kTmaStaticSmemReserve = 1024;

__device__ unsigned int g_wait_timeouts;

// Vector `v` (VEC bytes) of a row staged in shared memory, as 16-byte reads.
template <int VEC>
__device__ __forceinline__ Vec<VEC> ld_staged(const unsigned char* row, int v) {
  Vec<VEC> out;
  const uint4* p = reinterpret_cast<const uint4*>(row + static_cast<size_t>(v) * VEC);
#pragma unroll
  for (int k = 0; k < VEC / 16; ++k) {
    const uint4 q = p[k];
    out.w[4 * k] = q.x, out.w[4 * k + 1] = q.y, out.w[4 * k + 2] = q.z, out.w[4 * k + 3] = q.w;
  }
  return out;
}

template <typename T, int VEC, int VPT, bool RES>
__global__ void __launch_bounds__(cta_max_threads(VPT * VEC / 16)) rms_norm_tma_rows(RmsArgs a) {
  static_assert(VEC == 16 || VEC == 32, "rows are staged as 16-byte pieces");
  constexpr int EPV = Vec<VEC>::kElems;
  extern __shared__ __align__(128) unsigned char stage_mem[];
  __shared__ __align__(8) uint64_t full[kTmaMaxStages];
  __shared__ float warp_part[2][32];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int nwarps = nthreads >> 5;
  const int stages = a.rows_per_cta;
  const uint32_t row_bytes = static_cast<uint32_t>(a.nvec) * VEC;
  const uint32_t stage_bytes = (RES ? 2u : 1u) * row_bytes;
  const int64_t first = blockIdx.x;
  const int64_t step = gridDim.x;
  const int64_t count = first < a.rows ? (a.rows - 1 - first) / step + 1 : 0;
  uint16_t* out = static_cast<uint16_t*>(a.out);
  const uint64_t pol_stream = policy_evict_first();
  const uint64_t pol_keep = policy_evict_last();

  auto issue = [&](int64_t k, int s) {
    const int64_t row = first + k * step;
    const uint32_t bar = smem_u32(&full[s]);
    const uint32_t dst = smem_u32(stage_mem + static_cast<size_t>(s) * stage_bytes);
    mbar_arrive_expect_tx(bar, stage_bytes + (row == a.stall_row ? kStallBytes : 0u));
    bulk_load(dst, a.x + row * a.x_stride, row_bytes, bar, pol_stream);
    if constexpr (RES) bulk_load(dst + row_bytes, a.r + row * a.r_stride, row_bytes, bar, pol_stream);
  };

  pdl_wait();
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(smem_u32(&full[s]), 1);
    mbar_init_fence();
    for (int s = 0; s < stages && s < count; ++s) issue(s, s);
  }
  Vec<VEC> wv[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = tid + j * nthreads;
    if (v < a.nvec) wv[j] = ld_weight<VEC>(a.w + static_cast<int64_t>(v) * EPV, pol_keep);
  }
  __syncthreads();

  int s = 0;
  uint32_t parity = 0;
  for (int64_t k = 0; k < count; ++k) {
    const int64_t row = first + k * step;
    const bool arrived = mbar_wait_bounded(smem_u32(&full[s]), parity, a.wait_limit_ns);
    const unsigned char* xs = stage_mem + static_cast<size_t>(s) * stage_bytes;
    uint16_t* rr = RES ? a.r + row * a.r_stride : nullptr;
    Vec<VEC> xv[VPT];
    float a0 = 0.f, a1 = 0.f;
    if (arrived) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = tid + j * nthreads;
        if (v < a.nvec) {
          xv[j] = ld_staged<VEC>(xs, v);
          if constexpr (RES) {
            add_round<T, VEC>(xv[j], ld_staged<VEC>(xs + row_bytes, v), a0, a1);
          } else {
            square_sum<T, VEC>(xv[j], a0, a1);
          }
        }
      }
    }
    const float wsum = warp_sum(a0 + a1);
    if (lane == 0) warp_part[k & 1][warp] = wsum;
    // Every thread has read stage s (or some thread gave up waiting).
    if (__syncthreads_or(!arrived)) {
      if (tid == 0) {
        // Let this CTA's copies still in flight land before its shared memory
        // goes: wait (bounded) for every stage it issued and has not consumed.
        // A stalled row's phase is first given the bytes it was made to
        // expect beyond its copies, so it completes when they have landed.
        int ws = s;
        uint32_t wp = parity;
        for (int64_t j = k; j < count && j < k + stages; ++j) {
          if (first + j * step == a.stall_row) mbar_complete_tx(smem_u32(&full[ws]), kStallBytes);
          mbar_wait_bounded(smem_u32(&full[ws]), wp);
          if (++ws == stages) ws = 0, wp ^= 1u;
        }
        atomicAdd(&g_wait_timeouts, 1u);
      }
      return;
    }
    if constexpr (RES) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = tid + j * nthreads;
        if (v < a.nvec) st_global<VEC>(rr + static_cast<int64_t>(v) * EPV, xv[j]);
      }
    }
    if (tid == 0 && k + stages < count) {
      fence_proxy_async_smem();
      issue(k + stages, s);
    }
    const float total = warp_sum(lane < nwarps ? warp_part[k & 1][lane] : 0.f);
    const float inv = rsqrtf(fmaf(total, a.inv_hidden, a.eps));
    uint16_t* orow = out + row * a.out_stride;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = tid + j * nthreads;
      if (v < a.nvec)
        st_global<VEC>(orow + static_cast<int64_t>(v) * EPV, normalize<T, VEC>(xv[j], wv[j], inv));
    }
    if (++s == stages) s = 0, parity ^= 1u;
  }
  pdl_trigger();
}

}  // namespace hprn
