// Per-layer orthogonal rotation of head vectors, y = x @ R (or x @ R^T), in
// fp32 (backend.py:238-246 applies R_k to keys and queries, R_v to values and
// R_v^T to the attention output).  The reference runs these as fp32 library
// GEMMs on [tokens * heads, D] x [D, D]; here one kernel reads x in its own
// dtype, accumulates in fp32 FMAs over the D products and writes fp32 and/or
// the query dtype straight into strided destination rows, which also fuses
// the casts and copies around the GEMM.  One launch serves up to four
// segments (e.g. the step's queries, keys and values) that share the dtypes.
//
// CTA = 16 rows x 32 output columns of one segment, 256 threads.  The [D, 32]
// column block of R and the [16, D] row tile of x (transposed to [D, 16]) are
// staged in shared memory (48 KB at D = 256).  The reduction over k is split
// across the 8 warps (D / 8 products each); inside a warp, lane (rg, cg)
// accumulates a 4 x 4 register tile (rows 4 rg.., columns 4 cg..) from one
// 16-byte x load and one 16-byte R load per k, both single-wavefront.  The
// eight partial tiles are summed through shared memory in warp order.
#pragma once

#include "common.cuh"

namespace oscar {

constexpr int kRotRows = 16;
constexpr int kRotCols = 32;
constexpr int kRotMaxSegs = 4;

struct RotSeg {
  const void* x;
  int64_t rows, x_stride;
  int heads;  // rows r = token * heads + head: x at token * x_stride + head * D (outputs likewise)
  const float* rot;
  int transpose;
  void* out;
  int64_t out_stride;
  float* out_f32;
  int64_t out_f32_stride;
};

struct RotBatch {
  RotSeg seg[kRotMaxSegs];
  int tile_begin[kRotMaxSegs + 1];  // first row tile of each segment; tile_begin[n] = all tiles
  int n;
  int rot_early;  // 1: no rotation matrix was written by the launch in front (its loads may overlap it)
};

template <int D>
constexpr size_t rotate_smem_bytes() {
  return (size_t)(D * kRotCols + D * kRotRows) * sizeof(float) > (size_t)8 * kRotRows * kRotCols * sizeof(float)
             ? (size_t)(D * kRotCols + D * kRotRows) * sizeof(float)
             : (size_t)8 * kRotRows * kRotCols * sizeof(float);
}

// element offset of row r (token r / heads, head r % heads)
OSCAR_DEVINL int64_t rot_row(int64_t r, int heads, int64_t stride, int d) {
  if (heads == 1) return r * stride;
  const int64_t t = r / heads;
  return t * stride + (r - t * heads) * d;
}

template <typename T>
OSCAR_DEVINL void rot_store(T* p, float v) {
  *p = Elem<T>::from_f32(v);
}
template <>
OSCAR_DEVINL void rot_store<float>(float* p, float v) {
  *p = v;
}

// 16 bytes of x -> fp32 (8 elements for 16-bit types, 4 for fp32)
template <typename T>
struct RotIn {
  static constexpr int kPer16 = 8;
  static OSCAR_DEVINL void convert(const uint4& u, float* f) {
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_f32(e[i]);
  }
};
template <>
struct RotIn<float> {
  static constexpr int kPer16 = 4;
  static OSCAR_DEVINL void convert(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
};

template <typename InT, typename OutT, int D>
__global__ void __launch_bounds__(256) rotate_rows_kernel(const __grid_constant__ RotBatch b) {
  pdl_release();
  if (!b.rot_early) pdl_wait();
  extern __shared__ __align__(16) float rsm[];
  float* rblk = rsm;                 // [D][32]: R[k][c0 + j] (R^T: R[c0 + j][k])
  float* xt = rsm + D * kRotCols;    // [D][16]: x[r0 + r][k] at k * 16 + r
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int si = 0;
  while (si + 1 < b.n && (int)blockIdx.x >= b.tile_begin[si + 1]) ++si;
  const RotSeg& sg = b.seg[si];
  const int64_t r0 = (int64_t)((int)blockIdx.x - b.tile_begin[si]) * kRotRows;
  const int c0 = blockIdx.y * kRotCols;
  const InT* x = static_cast<const InT*>(sg.x);
  const float* rot = sg.rot;
  // every global load of the CTA is issued before the first shared-memory
  // store: one round trip instead of one per unrolled batch
  constexpr int kRLoads = D * kRotCols / 4 / 256;  // float4 of R per thread
  constexpr int kP = RotIn<InT>::kPer16;
  constexpr int kXChunks = kRotRows * D / kP;      // 16-byte chunks of the x tile
  constexpr int kXLoads = (kXChunks + 255) / 256;
  float4 rbuf[kRLoads];
#pragma unroll
  for (int u = 0; u < kRLoads; ++u) {
    const int i = tid + 256 * u;
    if (!sg.transpose) {
      // (k, 4 c4 .. 4 c4 + 3): a warp reads 4 rows x 128 B
      const int k = i >> 3, c4 = i & 7;
      rbuf[u] = *reinterpret_cast<const float4*>(rot + (int64_t)k * D + c0 + 4 * c4);
    } else {
      // R^T[k][c] = R[c][k]: a warp reads 8 rows c x 64 B along k
      const int rest = i >> 5;
      const int j = ((rest & 3) << 3) | (i & 7), k4 = ((rest >> 2) << 2) | ((i >> 3) & 3);
      rbuf[u] = *reinterpret_cast<const float4*>(rot + (int64_t)(c0 + j) * D + 4 * k4);
    }
  }
  // rotation matrices are layer constants: unless the launch in front wrote one
  // (rot_early = 0), their loads overlap that launch's tail (programmatic
  // dependent launch) and only the rows x wait for it
  pdl_wait();
  uint4 xbuf[kXLoads];
#pragma unroll
  for (int u = 0; u < kXLoads; ++u) {
    const int i = tid + 256 * u;
    const int r = i & (kRotRows - 1), kc = i >> 4;
    xbuf[u] = make_uint4(0u, 0u, 0u, 0u);
    if (i < kXChunks && r0 + r < sg.rows)
      xbuf[u] = *reinterpret_cast<const uint4*>(x + rot_row(r0 + r, sg.heads, sg.x_stride, D) + kP * kc);
  }
#pragma unroll
  for (int u = 0; u < kRLoads; ++u) {
    const int i = tid + 256 * u;
    const float4 v = rbuf[u];
    if (!sg.transpose) {
      const int k = i >> 3, c4 = i & 7;
      *reinterpret_cast<float4*>(rblk + k * kRotCols + 4 * c4) = v;
    } else {
      const int rest = i >> 5;
      const int j = ((rest & 3) << 3) | (i & 7), k4 = ((rest >> 2) << 2) | ((i >> 3) & 3);
      rblk[(4 * k4) * kRotCols + j] = v.x;
      rblk[(4 * k4 + 1) * kRotCols + j] = v.y;
      rblk[(4 * k4 + 2) * kRotCols + j] = v.z;
      rblk[(4 * k4 + 3) * kRotCols + j] = v.w;
    }
  }
#pragma unroll
  for (int u = 0; u < kXLoads; ++u) {
    const int i = tid + 256 * u;
    if (i < kXChunks) {
      const int r = i & (kRotRows - 1), kc = i >> 4;
      float f[kP];
      RotIn<InT>::convert(xbuf[u], f);
#pragma unroll
      for (int e = 0; e < kP; ++e) xt[(kP * kc + e) * kRotRows + r] = f[e];
    }
  }
  __syncthreads();

  constexpr int kSlice = D / 8;  // products per warp
  const int rg = lane >> 3, cg = lane & 7;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  const float* xp = xt + warp * kSlice * kRotRows + 4 * rg;
  const float* rp = rblk + warp * kSlice * kRotCols + 4 * cg;
#pragma unroll 8
  for (int kk = 0; kk < kSlice; ++kk) {
    const float4 xv = *reinterpret_cast<const float4*>(xp + kk * kRotRows);
    const float4 rv = *reinterpret_cast<const float4*>(rp + kk * kRotCols);
    const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, ra[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], ra[j], acc[i][j]);
  }
  __syncthreads();  // every warp is done with rblk / xt
  float* red = rsm;  // [8 warps][16 rows][32 cols]
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4*>(red + warp * kRotRows * kRotCols + (4 * rg + i) * kRotCols + 4 * cg) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  __syncthreads();
  const int r = tid >> 4, cq = 2 * (tid & 15);
  float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const float2 p = *reinterpret_cast<const float2*>(red + w * kRotRows * kRotCols + r * kRotCols + cq);
    s.x += p.x;
    s.y += p.y;
  }
  if (r0 + r < sg.rows) {
    const float v[2] = {s.x, s.y};
    OutT* out = static_cast<OutT*>(sg.out);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (out != nullptr) rot_store<OutT>(out + rot_row(r0 + r, sg.heads, sg.out_stride, D) + c0 + cq + j, v[j]);
      if (sg.out_f32 != nullptr) sg.out_f32[rot_row(r0 + r, sg.heads, sg.out_f32_stride, D) + c0 + cq + j] = v[j];
    }
  }
}

}  // namespace oscar
