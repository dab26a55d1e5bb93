// Per-layer rotation of large batches with fp32 FMAs, register-tiled: the
// same arithmetic class as rotate.cuh (every product and sum an fp32 FMA, each
// output one ordered chain over k), at a tile size that keeps the FMA pipe,
// not shared memory, the limit.
//
// CTA = ROWS (128 or 64) rows x 128 output columns of one segment, 256
// threads; thread (ty, tx) = (tid / 16, tid % 16) accumulates rows
// {4 ty + i, 64 + 4 ty + i} (only {4 ty + i} at ROWS 64) x columns
// {4 tx + j, 64 + 4 tx + j} over k in chunks of 32: x (converted to fp32,
// transposed to [k][row]) and R ([k][column]) are staged in shared memory,
// double-buffered, so each k costs four (three) 16-byte shared loads per 64
// (32) FMAs.  128-row tiles for long segments, 64-row tiles for mid-sized
// ones (twice the CTAs on the SMs), rotate.cuh's 16-row tiles below that.
#pragma once

#include "common.cuh"
#include "rotate.cuh"

namespace oscar {

constexpr int kRbCols = 128;
constexpr int kRbK = 32;
constexpr int kRbThreads = 256;

template <int ROWS>
struct RbSmem {
  float xs[2][kRbK][ROWS];     // x^T of the chunk
  float rs[2][kRbK][kRbCols];  // R rows of the chunk (columns c0 ..)
};

// one 16-byte chunk of x -> fp32 values (8 of a 16-bit type, 4 of fp32)
template <typename InT>
struct RbIn {
  static constexpr int kPer = 8;
  static OSCAR_DEVINL void convert(const uint4& u, float* f) {
    const InT* e = reinterpret_cast<const InT*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = Elem<InT>::to_f32(e[j]);
  }
};
template <>
struct RbIn<float> {
  static constexpr int kPer = 4;
  static OSCAR_DEVINL void convert(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
};

template <typename InT, typename OutT, int D, int ROWS>
__global__ void __launch_bounds__(kRbThreads, ROWS == 64 && sizeof(InT) == 2 ? 3 : 1) rotate_big_kernel(const __grid_constant__ RotBatch b) {
  static_assert(ROWS == 128 || ROWS == 64, "row tiles of 128 or 64");
  constexpr int kRg = ROWS / 64;  // groups of 4 rows per thread: rows 64 g + 4 ty + i
  constexpr int kUnroll = ROWS == 64 ? kRbK : 8;  // k-steps per unrolled body (64-row tiles: within 80 registers)
  pdl_release();
  if (!b.rot_early) pdl_wait();
  extern __shared__ __align__(16) uint8_t rb_raw[];
  RbSmem<ROWS>& sm = *reinterpret_cast<RbSmem<ROWS>*>(rb_raw);
  constexpr int kPer = RbIn<InT>::kPer;
  constexpr int kCpr = kRbK / kPer;                       // 16-byte chunks per row of a chunk
  constexpr int kXItems = ROWS * kCpr / kRbThreads;       // x chunks per thread per k-chunk
  constexpr int kRItems = kRbK * kRbCols / 4 / kRbThreads;  // float4 of R per thread per k-chunk
  constexpr int kChunks = D / kRbK;
  const int tid = threadIdx.x;
  int si = 0;
  while (si + 1 < b.n && (int)blockIdx.x >= b.tile_begin[si + 1]) ++si;
  const RotSeg& sg = b.seg[si];
  const int64_t r0 = (int64_t)((int)blockIdx.x - b.tile_begin[si]) * ROWS;
  const int c0 = blockIdx.y * kRbCols;
  const float* rot = sg.rot;

  // loaders: x chunk u of this thread = (row, 16-byte piece); R float4 u = (k, column group)
  auto load_r = [&](int kc, float4 (&rr)[kRItems]) {
#pragma unroll
    for (int u = 0; u < kRItems; ++u) {
      const int i = tid + kRbThreads * u;
      const int k = i / (kRbCols / 4), c4 = i % (kRbCols / 4);
      const int kk = kc * kRbK + k;
      if (!sg.transpose) {
        rr[u] = *reinterpret_cast<const float4*>(rot + (int64_t)kk * D + c0 + 4 * c4);
      } else {
        // R^T[kk][c] = R[c][kk]
        rr[u] = make_float4(rot[(int64_t)(c0 + 4 * c4) * D + kk], rot[(int64_t)(c0 + 4 * c4 + 1) * D + kk],
                            rot[(int64_t)(c0 + 4 * c4 + 2) * D + kk], rot[(int64_t)(c0 + 4 * c4 + 3) * D + kk]);
      }
    }
  };
  const InT* xsrc[kXItems];
  bool xlive[kXItems];
  pdl_wait();
#pragma unroll
  for (int u = 0; u < kXItems; ++u) {
    const int i = tid + kRbThreads * u;
    const int64_t row = r0 + i / kCpr;
    xlive[u] = row < sg.rows;
    xsrc[u] = static_cast<const InT*>(sg.x) + (xlive[u] ? rot_row(row, sg.heads, sg.x_stride, D) : 0) + kPer * (i % kCpr);
  }
  auto load_x = [&](int kc, uint4 (&xr)[kXItems]) {
#pragma unroll
    for (int u = 0; u < kXItems; ++u)
      xr[u] = xlive[u] ? *reinterpret_cast<const uint4*>(xsrc[u] + kc * kRbK) : make_uint4(0u, 0u, 0u, 0u);
  };
  auto store = [&](int buf, const uint4 (&xr)[kXItems], const float4 (&rr)[kRItems]) {
#pragma unroll
    for (int u = 0; u < kXItems; ++u) {
      const int i = tid + kRbThreads * u;
      const int row = i / kCpr, kb = kPer * (i % kCpr);
      float f[kPer];
      RbIn<InT>::convert(xr[u], f);
#pragma unroll
      for (int e = 0; e < kPer; ++e) sm.xs[buf][kb + e][row] = f[e];
    }
#pragma unroll
    for (int u = 0; u < kRItems; ++u) {
      const int i = tid + kRbThreads * u;
      const int k = i / (kRbCols / 4), c4 = i % (kRbCols / 4);
      *reinterpret_cast<float4*>(&sm.rs[buf][k][4 * c4]) = rr[u];
    }
  };

  const int ty = tid >> 4, tx = tid & 15;
  float acc[4 * kRg][8];
#pragma unroll
  for (int i = 0; i < 4 * kRg; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  {
    uint4 xr[kXItems];
    float4 rr[kRItems];
    load_x(0, xr);
    load_r(0, rr);
    store(0, xr, rr);
  }
  __syncthreads();
  for (int kc = 0; kc < kChunks; ++kc) {
    const int buf = kc & 1;
    uint4 xr[kXItems];
    float4 rr[kRItems];
    if (kc + 1 < kChunks) {
      load_x(kc + 1, xr);
      load_r(kc + 1, rr);
    }
    // the fragments of k-step k + 1 are loaded while k-step k computes (two
    // register slots): with one or two CTAs per SM the shared-memory latency
    // is not hidden by other warps
    float4 fx[2][kRg], fr[2][2];
    auto frag = [&](int k, float4 (&x)[kRg], float4 (&r)[2]) {
#pragma unroll
      for (int g = 0; g < kRg; ++g) x[g] = *reinterpret_cast<const float4*>(&sm.xs[buf][k][64 * g + 4 * ty]);
      r[0] = *reinterpret_cast<const float4*>(&sm.rs[buf][k][4 * tx]);
      r[1] = *reinterpret_cast<const float4*>(&sm.rs[buf][k][64 + 4 * tx]);
    };
    frag(0, fx[0], fr[0]);
#pragma unroll(kUnroll)
    for (int k = 0; k < kRbK; ++k) {
      if (k + 1 < kRbK) frag(k + 1, fx[(k + 1) & 1], fr[(k + 1) & 1]);
      float xv[4 * kRg];
#pragma unroll
      for (int g = 0; g < kRg; ++g) {
        const float4 xa = fx[k & 1][g];
        xv[4 * g] = xa.x;
        xv[4 * g + 1] = xa.y;
        xv[4 * g + 2] = xa.z;
        xv[4 * g + 3] = xa.w;
      }
      const float4 ra = fr[k & 1][0], rb = fr[k & 1][1];
      const float rv[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
#pragma unroll
      for (int i = 0; i < 4 * kRg; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(xv[i], rv[j], acc[i][j]);
    }
    if (kc + 1 < kChunks) store(buf ^ 1, xr, rr);
    __syncthreads();
  }
  OutT* out = static_cast<OutT*>(sg.out);
#pragma unroll
  for (int i = 0; i < 4 * kRg; ++i) {
    const int64_t row = r0 + 64 * (i / 4) + 4 * ty + (i % 4);
    if (row >= sg.rows) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = c0 + 64 * h + 4 * tx;
      if (out != nullptr) {
        OutT* o = out + rot_row(row, sg.heads, sg.out_stride, D) + col;
#pragma unroll
        for (int j = 0; j < 4; ++j) rot_store<OutT>(o + j, acc[i][4 * h + j]);
      }
      if (sg.out_f32 != nullptr)
        *reinterpret_cast<float4*>(sg.out_f32 + rot_row(row, sg.heads, sg.out_f32_stride, D) + col) =
            make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
    }
  }
}

}  // namespace oscar
