// Vector memory access and 16-bit float packing helpers for sm_100a.
//
// A "vector" is VEC bytes of one row: 32 (ld/st.global.v8.b32, the Blackwell
// 256-bit access), 16, 8, 4 or 2 bytes.  Elements are 16-bit (bf16 or fp16)
// and travel as raw bit patterns; arithmetic is fp32.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace hprn {

template <int VEC>
struct Vec {
  static constexpr int kWords = VEC / 4;  // 32-bit words
  static constexpr int kElems = VEC / 2;  // 16-bit elements
  uint32_t w[kWords];
};

template <>
struct Vec<2> {
  static constexpr int kWords = 0;
  static constexpr int kElems = 1;
  uint16_t h;
};

// ---------------------------------------------------------------------------
// L2 cache policies (createpolicy): streamed rows are read once, so they are
// marked evict_first; the weight row is re-read by every row and is kept with
// evict_last.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------
// Streaming loads: bypass L1 allocation, L2 evict_first.
template <int VEC>
__device__ __forceinline__ Vec<VEC> ld_stream(const void* p, uint64_t pol);

template <>
__device__ __forceinline__ Vec<32> ld_stream<32>(const void* p, uint64_t pol) {
  Vec<32> v;
  asm volatile(
      "ld.global.L1::no_allocate.L2::cache_hint.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
      : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
        "=r"(v.w[6]), "=r"(v.w[7])
      : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<16> ld_stream<16>(const void* p, uint64_t pol) {
  Vec<16> v;
  asm volatile("ld.global.L1::no_allocate.L2::cache_hint.v4.b32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<8> ld_stream<8>(const void* p, uint64_t pol) {
  Vec<8> v;
  asm volatile("ld.global.L1::no_allocate.L2::cache_hint.v2.b32 {%0,%1}, [%2], %3;"
               : "=r"(v.w[0]), "=r"(v.w[1])
               : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<4> ld_stream<4>(const void* p, uint64_t pol) {
  Vec<4> v;
  asm volatile("ld.global.L1::no_allocate.L2::cache_hint.b32 %0, [%1], %2;"
               : "=r"(v.w[0])
               : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<2> ld_stream<2>(const void* p, uint64_t pol) {
  Vec<2> v;
  asm volatile("ld.global.L1::no_allocate.L2::cache_hint.b16 %0, [%1], %2;"
               : "=h"(v.h)
               : "l"(p), "l"(pol));
  return v;
}

// ---------------------------------------------------------------------------
// Weight loads: read-only path, kept in L1 and (evict_last) in L2.
template <int VEC>
__device__ __forceinline__ Vec<VEC> ld_weight(const void* p, uint64_t pol);

template <>
__device__ __forceinline__ Vec<32> ld_weight<32>(const void* p, uint64_t pol) {
  Vec<32> v;
  asm volatile(
      "ld.global.nc.L1::evict_last.L2::cache_hint.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
      : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
        "=r"(v.w[6]), "=r"(v.w[7])
      : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<16> ld_weight<16>(const void* p, uint64_t pol) {
  Vec<16> v;
  asm volatile("ld.global.nc.L1::evict_last.L2::cache_hint.v4.b32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<8> ld_weight<8>(const void* p, uint64_t pol) {
  Vec<8> v;
  asm volatile("ld.global.nc.L1::evict_last.L2::cache_hint.v2.b32 {%0,%1}, [%2], %3;"
               : "=r"(v.w[0]), "=r"(v.w[1])
               : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<4> ld_weight<4>(const void* p, uint64_t pol) {
  Vec<4> v;
  asm volatile("ld.global.nc.L1::evict_last.L2::cache_hint.b32 %0, [%1], %2;"
               : "=r"(v.w[0])
               : "l"(p), "l"(pol));
  return v;
}

template <>
__device__ __forceinline__ Vec<2> ld_weight<2>(const void* p, uint64_t pol) {
  Vec<2> v;
  asm volatile("ld.global.nc.L1::evict_last.L2::cache_hint.b16 %0, [%1], %2;"
               : "=h"(v.h)
               : "l"(p), "l"(pol));
  return v;
}

// ---------------------------------------------------------------------------
// Plain loads that must observe this kernel's own earlier stores (the
// two-pass kernel re-reads the residual it just wrote): L1 is bypassed with
// .cg so the line comes from L2.
template <int VEC>
__device__ __forceinline__ Vec<VEC> ld_l2(const void* p);

template <>
__device__ __forceinline__ Vec<32> ld_l2<32>(const void* p) {
  Vec<32> v;
  asm volatile("ld.global.cg.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]),
                 "=r"(v.w[5]), "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p)
               : "memory");
  return v;
}

template <>
__device__ __forceinline__ Vec<16> ld_l2<16>(const void* p) {
  Vec<16> v;
  asm volatile("ld.global.cg.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "l"(p)
               : "memory");
  return v;
}

template <>
__device__ __forceinline__ Vec<8> ld_l2<8>(const void* p) {
  Vec<8> v;
  asm volatile("ld.global.cg.v2.b32 {%0,%1}, [%2];" : "=r"(v.w[0]), "=r"(v.w[1]) : "l"(p) : "memory");
  return v;
}

template <>
__device__ __forceinline__ Vec<4> ld_l2<4>(const void* p) {
  Vec<4> v;
  asm volatile("ld.global.cg.b32 %0, [%1];" : "=r"(v.w[0]) : "l"(p) : "memory");
  return v;
}

template <>
__device__ __forceinline__ Vec<2> ld_l2<2>(const void* p) {
  Vec<2> v;
  asm volatile("ld.global.cg.b16 %0, [%1];" : "=h"(v.h) : "l"(p) : "memory");
  return v;
}

// The same .cg load with an L2 cache policy (the two-pass kernel's last read
// of a row it staged in L2: evict_first).  Vector widths below 8 bytes take
// the plain load.
template <int VEC>
__device__ __forceinline__ Vec<VEC> ld_l2_hint(const void* p, uint64_t pol) {
  if constexpr (VEC == 32) {
    Vec<32> v;
    asm volatile("ld.global.cg.L2::cache_hint.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]),
                   "=r"(v.w[5]), "=r"(v.w[6]), "=r"(v.w[7])
                 : "l"(p), "l"(pol)
                 : "memory");
    return v;
  } else if constexpr (VEC == 16) {
    Vec<16> v;
    asm volatile("ld.global.cg.L2::cache_hint.v4.b32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(p), "l"(pol)
                 : "memory");
    return v;
  } else if constexpr (VEC == 8) {
    Vec<8> v;
    asm volatile("ld.global.cg.L2::cache_hint.v2.b32 {%0,%1}, [%2], %3;"
                 : "=r"(v.w[0]), "=r"(v.w[1])
                 : "l"(p), "l"(pol)
                 : "memory");
    return v;
  } else {
    return ld_l2<VEC>(p);
  }
}

// ---------------------------------------------------------------------------
// Stores.
template <int VEC>
__device__ __forceinline__ void st_global(void* p, const Vec<VEC>& v);

template <>
__device__ __forceinline__ void st_global<32>(void* p, const Vec<32>& v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.w[0]),
               "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]),
               "r"(v.w[7])
               : "memory");
}

template <>
__device__ __forceinline__ void st_global<16>(void* p, const Vec<16>& v) {
  asm volatile("st.global.v4.b32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
               "r"(v.w[2]), "r"(v.w[3])
               : "memory");
}

template <>
__device__ __forceinline__ void st_global<8>(void* p, const Vec<8>& v) {
  asm volatile("st.global.v2.b32 [%0], {%1,%2};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]) : "memory");
}

template <>
__device__ __forceinline__ void st_global<4>(void* p, const Vec<4>& v) {
  asm volatile("st.global.b32 [%0], %1;" ::"l"(p), "r"(v.w[0]) : "memory");
}

template <>
__device__ __forceinline__ void st_global<2>(void* p, const Vec<2>& v) {
  asm volatile("st.global.b16 [%0], %1;" ::"l"(p), "h"(v.h) : "memory");
}

// A store with an L2 cache policy (the two-pass kernel's rounded residual,
// which its second pass reads back: evict_last keeps it in L2 ahead of the
// streamed rows).  Vector widths below 8 bytes take the plain store.
template <int VEC>
__device__ __forceinline__ void st_global_hint(void* p, const Vec<VEC>& v, uint64_t pol) {
  if constexpr (VEC == 32) {
    asm volatile("st.global.L2::cache_hint.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8}, %9;" ::"l"(p),
                 "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]),
                 "r"(v.w[6]), "r"(v.w[7]), "l"(pol)
                 : "memory");
  } else if constexpr (VEC == 16) {
    asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "r"(v.w[0]),
                 "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "l"(pol)
                 : "memory");
  } else if constexpr (VEC == 8) {
    asm volatile("st.global.L2::cache_hint.v2.b32 [%0], {%1,%2}, %3;" ::"l"(p), "r"(v.w[0]),
                 "r"(v.w[1]), "l"(pol)
                 : "memory");
  } else {
    st_global<VEC>(p, v);
  }
}

// ---------------------------------------------------------------------------
// 16-bit float <-> fp32.  T is __nv_bfloat16 or __half.  Pairs use the packed
// conversions (cvt.rn.bf16x2.f32 / cvt.rn.f16x2.f32), round to nearest even.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w);

template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}

// {lo(a) * lo(b) + c.x, hi(a) * hi(b) + c.y} for 16-bit pairs a and b (bf16
// or fp16) with fp32 addends and results: sm_100's mixed-precision
// fma.rn.f32.{bf16,f16}.  The 16-bit operands widen to fp32 exactly and each
// element is rounded once, so the results are those of fmaf on the unpacked
// values, bit for bit, without the unpacking.
template <typename T>
__device__ __forceinline__ float2 fma_pair(uint32_t a, uint32_t b, float2 c);

template <>
__device__ __forceinline__ float2 fma_pair<__nv_bfloat16>(uint32_t a, uint32_t b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %2;\n\tmov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %4;\n\tfma.rn.f32.bf16 %1, ah, bh, %5;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "r"(a), "r"(b), "f"(c.x), "f"(c.y));
  return d;
}

template <>
__device__ __forceinline__ float2 fma_pair<__half>(uint32_t a, uint32_t b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %2;\n\tmov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %4;\n\tfma.rn.f32.f16 %1, ah, bh, %5;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "r"(a), "r"(b), "f"(c.x), "f"(c.y));
  return d;
}

// {lo(a) * lo(b), hi(a) * hi(b)} in fp32: exact, since a product of two
// 16-bit floats has at most 22 significant bits.  Adding -0 leaves every
// product, a zero's sign included, as fmul rounds it.
template <typename T>
__device__ __forceinline__ float2 mul_pair(uint32_t a, uint32_t b) {
  return fma_pair<T>(a, b, make_float2(-0.0f, -0.0f));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);

template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__device__ __forceinline__ float unpack1(uint16_t h);

template <>
__device__ __forceinline__ float unpack1<__nv_bfloat16>(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

template <>
__device__ __forceinline__ float unpack1<__half>(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

template <typename T>
__device__ __forceinline__ uint16_t pack1(float f);

template <>
__device__ __forceinline__ uint16_t pack1<__nv_bfloat16>(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

template <>
__device__ __forceinline__ uint16_t pack1<__half>(float f) {
  return __half_as_ushort(__float2half_rn(f));
}

// ---------------------------------------------------------------------------
// Eight e2m1 (NVFP4) codes of four fp32 pairs, converted and packed in
// registers: four cvt.rn.satfinite.e2m1x2.f32 assembled into one 32-bit word
// by a mov of the bytes, element order preserved (the first element in the
// lowest nibble).  The conversion is the one cuda_fp4.h uses: round to
// nearest even, saturating to the largest finite value.  Against the
// intrinsic's byte-by-byte shifts and ORs: 10.0 instead of 10.9 instructions
// per element for plain RMSNorm with NVFP4 output (4096 x 8192).
__device__ __forceinline__ uint32_t e2m1x8(float2 a, float2 b, float2 c, float2 d) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y), "f"(d.x), "f"(d.y));
  return r;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  pdl_wait() before the kernel's first
// global-memory load or store (only L2 prefetches come before it): blocks
// until the grid this one depends on (if it was launched that way) has
// completed and its memory is visible.  pdl_trigger() once a CTA's loads are
// issued (elementwise kernels, and row kernels in grids of more than one
// wave) or once its row reduction is done (single-wave row grids; after the
// last store is a launch knob): a following kernel launched with programmatic
// stream serialization may then be scheduled once every CTA of this grid has
// reached it (or exited), so its launch and its L2 prefetch overlap this
// grid's epilogue and drain; it still reads nothing before this grid has
// completed.  Triggering at kernel entry instead let the
// next grid's CTAs take SM slots and wait while this grid was still running:
// single-wave launches (decode batches) then took up to 40% longer than with no
// programmatic launch at all.  With no programmatic dependency both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Asks L2 to fetch [p, p + bytes) from DRAM: one bulk prefetch, which the
// TMA unit turns into line reads, so one thread covers a whole row slice at
// no register cost to the others.  Kernels issue it before pdl_wait() for the
// data they load first, so those DRAM reads overlap the preceding grid's
// drain and the dependency wait instead of following them.  It is a hint: it
// changes no register, shared-memory or memory contents, and the loads after
// the wait return the preceding grid's writes whether or not the lines were
// fetched before them (a prefetch is not a memory operation of the PTX memory
// consistency model).  The range is widened to whole 16-byte granules, as the
// instruction requires; a granule never straddles a page, so the widened
// range is mapped wherever [p, p + bytes) is.  bytes > 0.
__device__ __forceinline__ void prefetch_l2(const void* p, uint64_t bytes) {
  const uint64_t a = reinterpret_cast<uint64_t>(p);
  const uint64_t lo = a & ~uint64_t{15};
  const uint32_t n = static_cast<uint32_t>(((a + bytes + 15) & ~uint64_t{15}) - lo);
  asm volatile(
      "{\n\t.reg .u64 g;\n\tcvta.to.global.u64 g, %0;\n\t"
      "cp.async.bulk.prefetch.L2.global [g], %1;\n\t}" ::"l"(lo), "r"(n));
}

// No memory clobber: the trigger orders nothing (a dependent still waits for
// this grid's completion before it reads), so loads and stores stay free to
// move across it.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;");
}

}  // namespace hprn
