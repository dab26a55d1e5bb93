// Per-layer orthogonal rotation of head vectors, y = x @ R (or x @ R^T), in
// fp32 (backend.py:238-246 applies R_k to keys and queries, R_v to values and
// R_v^T to the attention output).  The reference runs these as fp32 library
// GEMMs on [tokens * heads, D] x [D, D]; here one kernel reads x in its own
// dtype, accumulates in fp32 FMAs over the D products and writes fp32 and/or
// the query dtype straight into strided destination rows, which also fuses
// the casts and copies around the GEMM.
//
// CTA = 16 rows x 32 output columns, 256 threads; the [D, 32] column block of
// R and the [16, D] row tile of x are staged in shared memory with 16-byte
// loads (48 KB at D = 256); thread t computes row t / 16 and columns
// 2 (t % 16), +1, each as two partial sums (even / odd k) to halve the
// dependent FMA chain.
#pragma once

#include "common.cuh"

namespace oscar {

constexpr int kRotRows = 16;
constexpr int kRotCols = 32;

template <typename T>
OSCAR_DEVINL void rot_store(T* p, float v) {
  *p = Elem<T>::from_f32(v);
}
template <>
OSCAR_DEVINL void rot_store<float>(float* p, float v) {
  *p = v;
}

// 8 elements of x (16 bytes for 16-bit types, two 16-byte loads for fp32) -> fp32
template <typename T>
OSCAR_DEVINL void rot_load8(const T* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_f32(e[i]);
}
template <>
OSCAR_DEVINL void rot_load8<float>(const float* p, float* f) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <typename InT, typename OutT, int D>
__global__ void __launch_bounds__(256) rotate_rows_kernel(const InT* __restrict__ x, int64_t x_stride, int64_t rows,
                                                          const float* __restrict__ rot, int transpose,
                                                          OutT* __restrict__ out, int64_t out_stride,
                                                          float* __restrict__ out_f32, int64_t out_f32_stride) {
  extern __shared__ __align__(16) float rsm[];
  float* rblk = rsm;                    // [D][32]: R[k][c0 + j] (R^T: R[c0 + j][k])
  float* xt = rsm + D * kRotCols;       // [16][D]
  const int tid = threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.x * kRotRows;
  const int c0 = blockIdx.y * kRotCols;
  if (!transpose) {
    // float4 (k, 4 c4 .. 4 c4 + 3): 8 per k row
#pragma unroll
    for (int i = tid; i < D * kRotCols / 4; i += 256) {
      const int k = i >> 3, c4 = i & 7;
      *reinterpret_cast<float4*>(rblk + k * kRotCols + 4 * c4) =
          *reinterpret_cast<const float4*>(rot + (int64_t)k * D + c0 + 4 * c4);
    }
  } else {
    // R^T[k][c] = R[c][k]: float4 along k of row c0 + j, scattered into column j
    // (consecutive threads take consecutive columns: conflict-free stores)
#pragma unroll
    for (int i = tid; i < D * kRotCols / 4; i += 256) {
      const int j = i & (kRotCols - 1), k4 = i / kRotCols;
      const float4 v = *reinterpret_cast<const float4*>(rot + (int64_t)(c0 + j) * D + 4 * k4);
      rblk[(4 * k4) * kRotCols + j] = v.x;
      rblk[(4 * k4 + 1) * kRotCols + j] = v.y;
      rblk[(4 * k4 + 2) * kRotCols + j] = v.z;
      rblk[(4 * k4 + 3) * kRotCols + j] = v.w;
    }
  }
#pragma unroll
  for (int i = tid; i < kRotRows * D / 8; i += 256) {
    const int r = i / (D / 8), k8 = i - r * (D / 8);
    float f[8];
    if (r0 + r < rows) {
      rot_load8<InT>(x + (r0 + r) * x_stride + 8 * k8, f);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = 0.0f;
    }
    *reinterpret_cast<float4*>(xt + r * D + 8 * k8) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(xt + r * D + 8 * k8 + 4) = make_float4(f[4], f[5], f[6], f[7]);
  }
  __syncthreads();
  const int r = tid >> 4, cq = 2 * (tid & 15);
  const float* xr = xt + r * D;
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [even / odd k][column]
#pragma unroll 8
  for (int k = 0; k < D; k += 2) {
    const float2 xv = *reinterpret_cast<const float2*>(xr + k);
    const float2 ra = *reinterpret_cast<const float2*>(rblk + k * kRotCols + cq);
    const float2 rb = *reinterpret_cast<const float2*>(rblk + (k + 1) * kRotCols + cq);
    acc[0][0] = fmaf(xv.x, ra.x, acc[0][0]);
    acc[0][1] = fmaf(xv.x, ra.y, acc[0][1]);
    acc[1][0] = fmaf(xv.y, rb.x, acc[1][0]);
    acc[1][1] = fmaf(xv.y, rb.y, acc[1][1]);
  }
  if (r0 + r < rows) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float v = acc[0][j] + acc[1][j];
      if (out != nullptr) rot_store<OutT>(out + (r0 + r) * out_stride + c0 + cq + j, v);
      if (out_f32 != nullptr) out_f32[(r0 + r) * out_f32_stride + c0 + cq + j] = v;
    }
  }
}

}  // namespace oscar
