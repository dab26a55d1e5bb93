// Shared device helpers for the OSCAR INT2 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define OSCAR_DEVINL __device__ __forceinline__

namespace oscar {

// Device-side bounds latch: kernels OR a bit in and skip the offending access.
// 1 = slot / block id out of range, 2 = block-table entry out of range,
// 8 = merge target row out of range.
__device__ unsigned int g_bounds_error;

OSCAR_DEVINL void flag_error(unsigned int bit) { atomicOr(&g_bounds_error, bit); }

// Programmatic dependent launch.  pdl_release lets the next kernel of the
// stream (launched with programmatic stream serialisation) start once every
// CTA of this grid has released; pdl_wait blocks until the previous kernel
// of the stream has completed and its memory is visible.  Both are no-ops
// for kernels launched without the attribute.
OSCAR_DEVINL void pdl_release() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
OSCAR_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// ---------------------------------------------------------------------------
// element types
template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static OSCAR_DEVINL __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
  static OSCAR_DEVINL float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  // history rounding chain of streaming_attention.py:124: fp32 -> fp16 -> bf16
  static OSCAR_DEVINL __nv_bfloat16 from_f16(__half h) { return __float2bfloat16_rn(__half2float(h)); }
};
template <> struct Elem<__half> {
  static OSCAR_DEVINL __half from_f32(float x) { return __float2half_rn(x); }
  static OSCAR_DEVINL float to_f32(__half x) { return __half2float(x); }
  static OSCAR_DEVINL __half from_f16(__half h) { return h; }
};

template <typename T>
OSCAR_DEVINL uint32_t pack2(T lo, T hi) {
  uint16_t a = *reinterpret_cast<uint16_t*>(&lo);
  uint16_t b = *reinterpret_cast<uint16_t*>(&hi);
  return (uint32_t)a | ((uint32_t)b << 16);
}

template <typename T>
OSCAR_DEVINL uint32_t pack2_f32(float lo, float hi) {
  return pack2<T>(Elem<T>::from_f32(lo), Elem<T>::from_f32(hi));
}

// fp16 bits (little-endian pair of bytes) -> float
OSCAR_DEVINL float f16_bits_to_f32(uint16_t bits) {
  __half h = *reinterpret_cast<__half*>(&bits);
  return __half2float(h);
}

// ---------------------------------------------------------------------------
// warp reductions
OSCAR_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
OSCAR_DEVINL float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// NaN-propagating max (torch.maximum semantics)
OSCAR_DEVINL float nan_max(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fffffff);
  return fmaxf(a, b);
}

// ---------------------------------------------------------------------------
// tensor-core and shared-memory PTX wrappers
OSCAR_DEVINL uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

OSCAR_DEVINL void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
OSCAR_DEVINL void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  static OSCAR_DEVINL void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<__half> {
  static OSCAR_DEVINL void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

}  // namespace oscar
