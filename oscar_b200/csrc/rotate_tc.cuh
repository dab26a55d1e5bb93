// Per-layer rotation of many head vectors on the tensor cores: y = x @ R (or
// x @ R^T) with tcgen05 kind::tf32 and split precision.
//
// The reference's rotations are fp32 GEMMs (backend.py:130-133, 360-373,
// 382); rotate.cuh computes them with fp32 FMAs, which at continuation sizes
// (15360 tokens x 24 query heads) takes as long as the attention.  Here R is
// split into R_hi = tf32(R) and R_lo = tf32(R - R_hi) and x into x_hi (+ x_lo
// for fp32 x; 16-bit x is exact in tf32), and the products x_hi R_hi +
// x_hi R_lo (+ x_lo R_hi) accumulate in fp32 in tensor memory: about 21 bits
// of R and of x enter the products, within a few fp32 ulps of the FMA kernel.
//
// Persistent CTAs: CTA (w, c) owns output columns [64 c, 64 c + 64) and the
// 128-row tiles w, w + gridDim.x, ... of the batch's segments (grid:
// min(tiles, SMs / column blocks) x D / 64); 288 threads:
//   warps 0-3 (loaders): load the CTA's 64 columns of R once (split, into
//     shared memory in the K-major no-swizzle layout of the B operand), then
//     stream each tile's x in slices of 32 k through a 3-slot ring
//     (consecutive lanes load consecutive 16-byte chunks of a row; converted /
//     split in registers; the next slice's loads in flight);
//   warp 4 (issuer): one elected lane issues, per slice, 4 k-steps of 2 or 3
//     MMAs (M 128, N 64, K 8) into the tile's accumulator (two in tensor
//     memory, alternating by tile) and commits the slot back to the loaders;
//   warps 5-8 (epilogue): read a finished accumulator (thread = row), free it
//     for the tile after next, write the outputs.
// Shared memory (D = 256): R_hi, R_lo 64 KB each; x slices 3 x (16 + 16) KB.
// Every wait is bounded; a timeout sets device error bit 16 and the CTA
// drains without writing.
#pragma once

#include "common.cuh"
#include "rotate.cuh"
#include "tc.cuh"

namespace oscar {

constexpr int kRtRows = 128;   // M: rows per CTA
constexpr int kRtCols = 64;    // N: output columns per CTA
constexpr int kRtK = 32;       // k per x slice
constexpr int kRtBufs = 3;     // x slice ring
constexpr int kRtThreads = 288;

template <int D>
struct RtSmem {
  uint8_t rhi[kRtCols * D * 4];             // B[n][k] = R[k][c0 + n]: (n/8)*(D/4*128) + (k/4)*128 + (n%8)*16 + (k%4)*4
  uint8_t rlo[kRtCols * D * 4];
  uint8_t xhi[kRtBufs][kRtRows * kRtK * 4];  // A[m][k]: (m/8)*1024 + (k/4)*128 + (m%8)*16 + (k%4)*4
  uint8_t xlo[kRtBufs][kRtRows * kRtK * 4];
  unsigned long long bar_full[kRtBufs], bar_empty[kRtBufs], bar_done[2], bar_free[2];
  uint32_t tmem;
  int abort;
};

OSCAR_DEVINL float rt_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// D[tmem] (+)= A[smem] * B[smem], kind::tf32
OSCAR_DEVINL void rt_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 32 consecutive outputs of a row (16-byte aligned): 16-byte stores
template <typename OutT>
OSCAR_DEVINL void rt_store32(OutT* o, const uint32_t (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = pack2<OutT>(Elem<OutT>::from_f32(__uint_as_float(v[8 * j + 2 * i])),
                         Elem<OutT>::from_f32(__uint_as_float(v[8 * j + 2 * i + 1])));
    reinterpret_cast<uint4*>(o)[j] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}
template <>
OSCAR_DEVINL void rt_store32<float>(float* o, const uint32_t (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    reinterpret_cast<float4*>(o)[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                  __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
}

// one 16-byte chunk of x -> fp32 values (8 of a 16-bit type, 4 of fp32)
template <typename InT>
struct RtLoad {
  static constexpr int kPer = 8;
  static OSCAR_DEVINL void convert(const uint4& u, float* f) {
    const InT* e = reinterpret_cast<const InT*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = Elem<InT>::to_f32(e[j]);
  }
};
template <>
struct RtLoad<float> {
  static constexpr int kPer = 4;
  static OSCAR_DEVINL void convert(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
};

template <typename InT, typename OutT, int D>
__global__ void __launch_bounds__(kRtThreads, 1) rotate_tc_kernel(const __grid_constant__ RotBatch b) {
  pdl_release();
  extern __shared__ __align__(1024) uint8_t rt_raw[];
  RtSmem<D>& sm = *reinterpret_cast<RtSmem<D>*>(rt_raw);
  constexpr bool kSplitX = std::is_same<InT, float>::value;
  constexpr int kSlices = D / kRtK;
  constexpr uint32_t kSboR = (uint32_t)(D / 4) * 128;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = b.tile_begin[b.n];
  const int c0 = blockIdx.y * kRtCols;
  const uint32_t b_full = smem_u32(&sm.bar_full[0]), b_empty = smem_u32(&sm.bar_empty[0]),
                 b_done = smem_u32(&sm.bar_done[0]), b_free = smem_u32(&sm.bar_free[0]);
  auto wait = [&](uint32_t bar, uint32_t parity) {
    if (tc::mbar_try(bar, parity)) return;
    if (*reinterpret_cast<volatile int*>(&sm.abort)) return;
    if (!tc::mbar_wait(bar, parity)) {
      *reinterpret_cast<volatile int*>(&sm.abort) = 1;
      flag_error(16u);
    }
  };
  // segment of a tile and its first row
  auto locate = [&](int tile, int& si, int64_t& r0) {
    si = 0;
    while (si + 1 < b.n && tile >= b.tile_begin[si + 1]) ++si;
    r0 = (int64_t)(tile - b.tile_begin[si]) * kRtRows;
  };

  if (warp == 4) {
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kRtBufs; ++i) {
        tc::mbar_init(b_full + 8 * i, 4);   // the four loader warps
        tc::mbar_init(b_empty + 8 * i, 1);  // the MMA commit
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        tc::mbar_init(b_done + 8 * i, 1);  // the tile's last commit
        tc::mbar_init(b_free + 8 * i, 4);  // the four epilogue warps
      }
      sm.abort = 0;
      tc::mbar_fence_init();
    }
    tc::tmem_alloc(smem_u32(&sm.tmem), 2 * kRtCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sm.tmem;

  if (warp < 4) {
    // ---- R columns [c0, c0 + 64), split, as B[n][k] (K-major).  Unless the launch in
    // front may have written a rotation, these loads overlap its tail.  (Every segment
    // of a batch shares one rotation layout; the CTA's tiles may span segments with
    // different matrices, so R is reloaded when the segment changes.)
    if (!b.rot_early) pdl_wait();
    const float* cur_rot = nullptr;
    auto load_r = [&](const RotSeg& g) {
      const float* rot = g.rot;
      constexpr int kItems = kRtCols * (D / 4) / 128;  // (n, k4) items per thread
      constexpr int kBatch = 8;
#pragma unroll 1
      for (int i0 = 0; i0 < kItems; i0 += kBatch) {
        float r[kBatch][4];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int i = tid + 128 * (i0 + u);
          const int n = i & (kRtCols - 1), k4 = i / kRtCols;
          if (!g.transpose) {
            // B[n][k] = R[k][c0 + n]: lanes read consecutive n of a row of R
#pragma unroll
            for (int j = 0; j < 4; ++j) r[u][j] = rot[(int64_t)(4 * k4 + j) * D + c0 + n];
          } else {
            // B[n][k] = R^T[k][c0 + n] = R[c0 + n][k]
            const float4 q = *reinterpret_cast<const float4*>(rot + (int64_t)(c0 + n) * D + 4 * k4);
            r[u][0] = q.x;
            r[u][1] = q.y;
            r[u][2] = q.z;
            r[u][3] = q.w;
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int i = tid + 128 * (i0 + u);
          const int n = i & (kRtCols - 1), k4 = i / kRtCols;
          float h[4], l[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            h[j] = rt_tf32(r[u][j]);
            l[j] = rt_tf32(r[u][j] - h[j]);
          }
          const uint32_t off = (uint32_t)(n >> 3) * kSboR + (uint32_t)k4 * 128 + (uint32_t)(n & 7) * 16;
          *reinterpret_cast<float4*>(sm.rhi + off) = make_float4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<float4*>(sm.rlo + off) = make_float4(l[0], l[1], l[2], l[3]);
        }
      }
      cur_rot = rot;
    };
    // x slices: thread tid loads 16-byte chunks (4 fp32 / 8 16-bit values of k) of
    // rows tid / kCpr + (128 / kCpr) u, so that consecutive lanes read consecutive
    // chunks of one row (kCpr chunks = one 32-k slice of a row)
    constexpr int kPer = RtLoad<InT>::kPer;         // values per 16-byte chunk
    constexpr int kCpr = kRtK / kPer;               // chunks per row of a slice
    constexpr int kItems = kRtRows * kCpr / 128;    // chunks per thread per slice
    const int cidx = tid % kCpr;
    int g = 0;  // slices issued by this CTA
    bool first = true;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      int si;
      int64_t r0;
      locate(tile, si, r0);
      const RotSeg& sg = b.seg[si];
      if (sg.rot != cur_rot) {
        // a new matrix: the slots that hold the old one must be consumed first
        for (int q = max(0, g - kRtBufs); q < g; ++q) wait(b_empty + 8 * (q % kRtBufs), (q / kRtBufs) & 1);
        load_r(sg);
      }
      if (first) {
        pdl_wait();
        first = false;
      }
      const InT* src[kItems];
      bool live[kItems];
#pragma unroll
      for (int u = 0; u < kItems; ++u) {
        const int64_t row = r0 + tid / kCpr + (128 / kCpr) * u;
        live[u] = row < sg.rows;
        src[u] = static_cast<const InT*>(sg.x) + (live[u] ? rot_row(row, sg.heads, sg.x_stride, D) : 0) + kPer * cidx;
      }
      uint4 cur[kItems];
#pragma unroll
      for (int u = 0; u < kItems; ++u) cur[u] = live[u] ? *reinterpret_cast<const uint4*>(src[u]) : make_uint4(0, 0, 0, 0);
      for (int s = 0; s < kSlices; ++s, ++g) {
        uint4 nxt[kItems];
        if (s + 1 < kSlices) {
#pragma unroll
          for (int u = 0; u < kItems; ++u)
            nxt[u] = live[u] ? *reinterpret_cast<const uint4*>(src[u] + (s + 1) * kRtK) : make_uint4(0, 0, 0, 0);
        }
        const int slot = g % kRtBufs;
        if (g >= kRtBufs) wait(b_empty + 8 * slot, ((g / kRtBufs) - 1) & 1);
#pragma unroll
        for (int u = 0; u < kItems; ++u) {
          const int m = tid / kCpr + (128 / kCpr) * u;
          float f[kPer];
          RtLoad<InT>::convert(cur[u], f);
#pragma unroll
          for (int c = 0; c < kPer / 4; ++c) {
            const int k4 = cidx * (kPer / 4) + c;
            float h[4], l[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              h[j] = kSplitX ? rt_tf32(f[4 * c + j]) : f[4 * c + j];
              l[j] = kSplitX ? rt_tf32(f[4 * c + j] - h[j]) : 0.0f;
            }
            const uint32_t off = (uint32_t)(m >> 3) * 1024 + (uint32_t)k4 * 128 + (uint32_t)(m & 7) * 16;
            *reinterpret_cast<float4*>(sm.xhi[slot] + off) = make_float4(h[0], h[1], h[2], h[3]);
            if (kSplitX) *reinterpret_cast<float4*>(sm.xlo[slot] + off) = make_float4(l[0], l[1], l[2], l[3]);
          }
        }
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(b_full + 8 * slot);
        if (s + 1 < kSlices) {
#pragma unroll
          for (int u = 0; u < kItems; ++u) cur[u] = nxt[u];
        }
      }
    }
    // every commit to the ring is complete before the CTA exits
    for (int q = max(0, g - kRtBufs); q < g; ++q) wait(b_empty + 8 * (q % kRtBufs), (q / kRtBufs) & 1);
  } else if (warp == 4) {
    // ---- MMA issuer
    constexpr uint32_t idesc = tc::instr_desc(2u, 0, 0, kRtRows, kRtCols);  // tf32 x tf32 -> f32
    const uint64_t dr_hi = tc::smem_desc(smem_u32(sm.rhi), 128, kSboR);
    const uint64_t dr_lo = tc::smem_desc(smem_u32(sm.rlo), 128, kSboR);
    int g = 0, t = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++t) {
      const int acc = t & 1;
      if (t >= 2) wait(b_free + 8 * acc, ((t >> 1) - 1) & 1);  // the epilogue read tile t - 2
      tc::tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(acc * kRtCols);
      for (int s = 0; s < kSlices; ++s, ++g) {
        const int slot = g % kRtBufs;
        wait(b_full + 8 * slot, (g / kRtBufs) & 1);
        tc::tc_fence_after();
        const uint64_t dxh = tc::smem_desc(smem_u32(sm.xhi[slot]), 128, 1024);
        const uint64_t dxl = tc::smem_desc(smem_u32(sm.xlo[slot]), 128, 1024);
        if (tc::elect_one()) {
#pragma unroll
          for (int j = 0; j < kRtK / 8; ++j) {
            // k-step j of the slice: 2 core matrices (256 bytes) into x, and
            // (s * 32 + 8 j) / 4 core matrices into R
            const uint64_t ax = (uint64_t)(16 * j), br = (uint64_t)((s * kRtK + 8 * j) / 4 * 8);
            rt_mma(d, dxh + ax, dr_hi + br, idesc, (s | j) != 0 ? 1u : 0u);
            rt_mma(d, dxh + ax, dr_lo + br, idesc, 1u);
            if (kSplitX) rt_mma(d, dxl + ax, dr_hi + br, idesc, 1u);
          }
          tc::mma_commit(b_empty + 8 * slot);
          if (s + 1 == kSlices) tc::mma_commit(b_done + 8 * acc);
        }
        __syncwarp();
      }
    }
  } else {
    // ---- epilogue warps 5-8: TMEM lane quarter (warp % 4), thread = row
    const int q = warp & 3;
    const int m = 32 * q + lane;
    int t = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++t) {
      int si;
      int64_t r0;
      locate(tile, si, r0);
      const RotSeg& sg = b.seg[si];
      const int acc = t & 1;
      wait(b_done + 8 * acc, (t >> 1) & 1);
      tc::tc_fence_after();
      uint32_t v[2][32];
      tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * kRtCols), v[0]);
      tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * kRtCols) + 32, v[1]);
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(b_free + 8 * acc);
      const int64_t row = r0 + m;
      if (row < sg.rows && !*reinterpret_cast<volatile int*>(&sm.abort)) {
        OutT* out = static_cast<OutT*>(sg.out);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = c0 + 32 * h;
          if (out != nullptr) rt_store32<OutT>(out + rot_row(row, sg.heads, sg.out_stride, D) + col, v[h]);
          if (sg.out_f32 != nullptr)
            rt_store32<float>(sg.out_f32 + rot_row(row, sg.heads, sg.out_f32_stride, D) + col, v[h]);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 4) tc::tmem_dealloc(tmem, 2 * kRtCols);
}

}  // namespace oscar
