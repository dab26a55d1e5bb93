// K2/K3 streaming attention over paged INT2 history, split-KV combine, K4 merge.
//
// Semantics: kernels/streaming_attention.py:134-196 (streaming_attention_ref)
// and kernels/slab_attention.py:376-476 (slab_attention).  Keys of request r
// are positions [0, seq): p < prefix come from the packed cache (an owner-tag
// hit reads the fp32 staging arena instead, streaming_attention.py:116-121),
// p >= prefix from the current chunk k_new/v_new.  History values take the
// reference's rounding chain value -> fp16 -> query dtype
// (streaming_attention.py:124).  Query i of the request sees keys
// [0, seq - q_len + i] (right-aligned causal, slab_attention.py:62-92).
//
// Work unit (CTA): (request, q-block, kv split) x kv-head.  A q-block packs
// `tpb` query tokens x G query heads of one kv-head as rows, so every dequantized
// key tile is shared by the whole GQA group.  NW warps each own 16 rows.
// Key tiles of 64 tokens are dequantized once into shared memory (XOR-swizzled
// 16-byte chunks), then S = Q K^T (query dtype) and O += P V (fp16 P and V)
// run on mma.sync with fp32 accumulation and an exp2-domain online softmax.
#pragma once

#include "common.cuh"

namespace oscar {

constexpr int kKT = 64;          // keys per tile
constexpr int kPlanReqs = 64;    // requests per launch (the plan travels by value)

struct AttnPlan {
  int num_req;
  int total_items;       // CTAs along x
  int total_merge_rows;  // rows to combine (requests with splits > 1)
  int tpb;               // query tokens per q-block
  int rows;              // rows per q-block (16 * NW)
  int req_id[kPlanReqs];
  int item_begin[kPlanReqs + 1];
  int merge_begin[kPlanReqs + 1];
  int part_begin[kPlanReqs + 1];
  int q_start[kPlanReqs];
  int q_len[kPlanReqs];
  int seq[kPlanReqs];
  int prefix[kPlanReqs];
  int splits[kPlanReqs];
  int chunk[kPlanReqs];
  int eff_tile[kPlanReqs + 1];  // continuation pre-pass: first 64-key tile of each request in AttnArgs::eff
};

struct AttnArgs {
  const void* q;
  const void* k_new;
  const void* v_new;
  int hq, hk, group;
  const uint8_t* kc;
  const uint8_t* vc;
  int64_t num_blocks;
  int bs;
  int64_t ksb, kst, ksh, vsb, vst, vsh;
  const int32_t* bt;
  int64_t bt_stride;
  float scale_log2;  // softmax scale * log2(e)
  const float* stage_k;
  const float* stage_v;
  const int64_t* owner;
  int64_t stage_rows;
  float* out;
  float* lse;
  float* part_o;
  float* part_lse;
  uint8_t* eff;  // continuation pre-pass output (tile layout of cont_tc.cuh), or nullptr
};

OSCAR_DEVINL int find_bucket(const int* begin, int n, int x) {
  int lo = 0, hi = n;  // last i with begin[i] <= x
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (begin[mid] <= x) lo = mid; else hi = mid;
  }
  return lo;
}

// 8 INT2 codes (little-endian 16 bits) -> 8 values of T via the exact chain
// fp32(code*scale + zero) -> fp16 -> T   (format.py:91-96 + streaming_attention.py:124)

// bf16/fp16 value of the reference chain -> fp16 operand of the P.V product.
// History and staged values went through fp16, so this is exact for them
// (bf16 rounding can only reach 65536 from >= 65280: clamped to the fp16 max).
template <typename T>
OSCAR_DEVINL uint32_t to_f16x2(uint32_t w) {
  T lo, hi;
  *reinterpret_cast<uint16_t*>(&lo) = (uint16_t)(w & 0xffffu);
  *reinterpret_cast<uint16_t*>(&hi) = (uint16_t)(w >> 16);
  const float a = fminf(fmaxf(Elem<T>::to_f32(lo), -65504.0f), 65504.0f);
  const float b = fminf(fmaxf(Elem<T>::to_f32(hi), -65504.0f), 65504.0f);
  return pack2<__half>(__float2half_rn(a), __float2half_rn(b));
}

template <typename T>
OSCAR_DEVINL uint4 to_f16x8(uint4 v) {
  return make_uint4(to_f16x2<T>(v.x), to_f16x2<T>(v.y), to_f16x2<T>(v.z), to_f16x2<T>(v.w));
}

template <typename T>
OSCAR_DEVINL uint4 staged8(const float* src) {
  const float4 a = *reinterpret_cast<const float4*>(src);
  const float4 b = *reinterpret_cast<const float4*>(src + 4);
  const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = pack2<T>(Elem<T>::from_f16(__float2half_rn(f[2 * i])), Elem<T>::from_f16(__float2half_rn(f[2 * i + 1])));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

OSCAR_DEVINL uint16_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// Fill one 64-key tile of K (type T) and V (fp16) in shared memory (swizzled)
// for keys [kt0, kt_end).  Phase 1 looks each key up once (block table,
// staging owner tag) into s_info; phase 2 gives a thread one (key, 64-dim
// group): a 16-byte load of K codes, one of V codes and one 8-byte load of the
// slot's scale / zero words for an INT2 key, or the key's fp32 staged rows,
// or its bf16/fp16 current-chunk rows.
constexpr int64_t kTileNone = INT64_MIN;  // zero fill: past the tile end or a bad block
constexpr int64_t kTileNew = -1;          // current-chunk key; <= -2: staged (-2 - seat); >= 0: INT2 slot

template <typename T>
OSCAR_DEVINL void tile_lut(uint32_t meta_sz, T (&lut)[4]) {
  const float sc = f16_bits_to_f32(meta_sz & 0xffffu), zr = f16_bits_to_f32(meta_sz >> 16);
#pragma unroll
  for (int c = 0; c < 4; ++c) lut[c] = Elem<T>::from_f16(__float2half_rn(__fadd_rn(__fmul_rn((float)c, sc), zr)));
}

template <int D, typename T, int NW>
OSCAR_DEVINL void load_kv_tile(const AttnArgs& a, T* sK, __half* sV, int kt0, int kt_end, int req, int h,
                               int q_start, int prefix, int64_t* s_info) {
  constexpr int G64 = D / 64;  // 64-dim groups per key
  const int tid = threadIdx.x;
  for (int r = tid; r < kKT; r += NW * 32) {
    const int p = kt0 + r;
    int64_t info = kTileNone;
    if (p < kt_end) {
      if (p < prefix) {
        const int pg = p / a.bs, off = p - pg * a.bs;
        const int64_t blk = a.bt[(int64_t)req * a.bt_stride + pg];
        if (blk < 0 || blk >= a.num_blocks) {
          flag_error(2u);
        } else {
          info = blk * a.bs + off;
          if (a.owner != nullptr) {
            const int64_t seat = (blk % a.stage_rows) * a.bs + off;
            if (a.owner[seat] == blk) info = -2 - seat;
          }
        }
      } else {
        info = kTileNew;
      }
    }
    s_info[r] = info;
  }
  __syncthreads();
  for (int it = tid; it < kKT * G64; it += NW * 32) {
    const int r = it / G64, g = it - (it / G64) * G64;
    const int64_t info = s_info[r];
    T* krow = sK + r * D;
    __half* vrow = sV + r * D;
    auto put = [&](int i, uint4 kw, uint4 vw) {  // 8-dim chunk 8 g + i
      const int sw = ((8 * g + i) ^ (r & 7)) * 8;
      *reinterpret_cast<uint4*>(krow + sw) = kw;
      *reinterpret_cast<uint4*>(vrow + sw) = vw;
    };
    if (info == kTileNone) {
#pragma unroll
      for (int i = 0; i < 8; ++i) put(i, make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0));
    } else if (info >= 0) {
      const int64_t blk = info / a.bs, off = info - (info / a.bs) * a.bs;
      const uint8_t* ks = a.kc + blk * a.ksb + off * a.kst + (int64_t)h * a.ksh;
      const uint8_t* vs = a.vc + blk * a.vsb + off * a.vst + (int64_t)h * a.vsh;
      uint2 meta;  // K scale, K zero, V scale, V zero
      uint4 kc, vc;
      if (((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs)) & 15) == 0) {
        meta = *reinterpret_cast<const uint2*>(ks);
        kc = *reinterpret_cast<const uint4*>(ks + 32 + 16 * g);
        vc = *reinterpret_cast<const uint4*>(vs + 16 * g);
      } else {
        // caches at an address or stride that is not 16-byte aligned: 16-bit reads
        auto w2 = [](const uint8_t* q) { return (uint32_t)ld_u16(q) | ((uint32_t)ld_u16(q + 2) << 16); };
        meta = make_uint2(w2(ks), w2(ks + 4));
        kc = make_uint4(w2(ks + 32 + 16 * g), w2(ks + 36 + 16 * g), w2(ks + 40 + 16 * g), w2(ks + 44 + 16 * g));
        vc = make_uint4(w2(vs + 16 * g), w2(vs + 4 + 16 * g), w2(vs + 8 + 16 * g), w2(vs + 12 + 16 * g));
      }
      T klut[4], vlut[4];
      tile_lut<T>(meta.x, klut);
      tile_lut<T>(meta.y, vlut);
      __half vl[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) vl[c] = __float2half_rn(fminf(fmaxf(Elem<T>::to_f32(vlut[c]), -65504.0f), 65504.0f));
      const uint32_t kws[4] = {kc.x, kc.y, kc.z, kc.w}, vws[4] = {vc.x, vc.y, vc.z, vc.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t kcode = (kws[i >> 1] >> (16 * (i & 1))) & 0xffffu;
        const uint32_t vcode = (vws[i >> 1] >> (16 * (i & 1))) & 0xffffu;
        uint32_t kw[4], vw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          kw[e] = pack2<T>(klut[(kcode >> (4 * e)) & 3u], klut[(kcode >> (4 * e + 2)) & 3u]);
          vw[e] = pack2<__half>(vl[(vcode >> (4 * e)) & 3u], vl[(vcode >> (4 * e + 2)) & 3u]);
        }
        put(i, make_uint4(kw[0], kw[1], kw[2], kw[3]), make_uint4(vw[0], vw[1], vw[2], vw[3]));
      }
    } else if (info == kTileNew) {
      const int64_t t = (int64_t)q_start + (kt0 + r - prefix);
      const int64_t base = (t * a.hk + h) * (int64_t)D + 64 * g;
      const uint4* kn = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.k_new) + base);
      const uint4* vn = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.v_new) + base);
#pragma unroll 4
      for (int i = 0; i < 8; ++i) put(i, kn[i], to_f16x8<T>(vn[i]));
    } else {  // staged: info = -2 - seat
      const int64_t base = ((-2 - info) * a.hk + h) * (int64_t)D + 64 * g;
#pragma unroll 2
      for (int i = 0; i < 8; ++i)
        put(i, staged8<T>(a.stage_k + base + 8 * i), to_f16x8<T>(staged8<T>(a.stage_v + base + 8 * i)));
    }
  }
}

template <int D, typename T, int NW>
__global__ void __launch_bounds__(NW * 32) paged_attn_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p) {
  constexpr int ROWS = 16 * NW;
  constexpr int NCH = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int64_t s_info[kKT];  // per-key lookups of the tile being loaded
  T* sQ = reinterpret_cast<T*>(smem);
  T* sK = sQ + ROWS * D;
  __half* sV = reinterpret_cast<__half*>(sK + kKT * D);

  const int item = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ri = find_bucket(p.item_begin, p.num_req, item);
  const int local = item - p.item_begin[ri];
  const int S = p.splits[ri];
  const int nqb = (p.item_begin[ri + 1] - p.item_begin[ri]) / S;
  const int qb = nqb - 1 - local / S;  // later (heavier) q-blocks first
  const int sp = local - (local / S) * S;
  const int req = p.req_id[ri];
  const int q_start = p.q_start[ri], qlen = p.q_len[ri], seq = p.seq[ri], prefix = p.prefix[ri];
  const int G = a.group;
  const int tok0 = qb * p.tpb;
  const int ntok = min(p.tpb, qlen - tok0);
  const int nrows = ntok * G;
  const int kv_hi_block = seq - qlen + tok0 + ntok;
  const int lo = sp * p.chunk[ri];
  const int hi = min(lo + p.chunk[ri], kv_hi_block);

  // Q rows -> shared memory (row = token * G + head-in-group)
  for (int idx = tid; idx < ROWS * NCH; idx += NW * 32) {
    const int row = idx / NCH, ch = idx - (idx / NCH) * NCH;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (row < nrows) {
      const int tl = row / G, hg = row - (row / G) * G;
      const T* src = reinterpret_cast<const T*>(a.q) +
                     ((int64_t)(q_start + tok0 + tl) * a.hq + (int64_t)h * G + hg) * D + ch * 8;
      val = *reinterpret_cast<const uint4*>(src);
    }
    *reinterpret_cast<uint4*>(sQ + row * D + ((ch ^ (row & 7)) * 8)) = val;
  }

  // per-thread rows g and g+8 of this warp's 16
  int lim[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = warp * 16 + (lane >> 2) + 8 * r;
    if (row < nrows) {
      const int tl = row / G;
      lim[r] = min(seq - qlen + tok0 + tl + 1, hi);
    } else {
      lim[r] = -1;
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};

  for (int kt0 = lo; kt0 < hi; kt0 += kKT) {
    __syncthreads();
    load_kv_tile<D, T, NW>(a, sK, sV, kt0, min(kt0 + kKT, hi), req, h, q_start, prefix, s_info);
    __syncthreads();

    float s[kKT / 8][4];
#pragma unroll
    for (int i = 0; i < kKT / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll 4
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t af[4];
      {
        const int row = warp * 16 + (lane & 15);
        const int ch = kk * 2 + (lane >> 4);
        ldmatrix_x4(smem_u32(sQ + row * D + ((ch ^ (row & 7)) * 8)), af[0], af[1], af[2], af[3]);
      }
#pragma unroll
      for (int j = 0; j < kKT / 16; ++j) {
        uint32_t b0, b1, b2, b3;
        const int key = j * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = kk * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(smem_u32(sK + key * D + ((ch ^ (key & 7)) * 8)), b0, b1, b2, b3);
        Mma<T>::run(s[2 * j], af, b0, b1);
        Mma<T>::run(s[2 * j + 1], af, b2, b3);
      }
    }

    // mask + online softmax (log2 domain)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < kKT / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const int key = kt0 + nt * 8 + 2 * (lane & 3) + (e & 1);
        const float v = (key < lim[r]) ? s[nt][e] * a.scale_log2 : -INFINITY;
        s[nt][e] = v;
        mx[r] = fmaxf(mx[r], v);
      }
    float muse[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      muse[r] = (m_new == -INFINITY) ? 0.0f : m_new;
      const float alpha = exp2f(m_run[r] - muse[r]);
      m_run[r] = m_new;
      l_run[r] *= alpha;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][2 * r] *= alpha;
        o[i][2 * r + 1] *= alpha;
      }
    }
#pragma unroll
    for (int nt = 0; nt < kKT / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float pv = exp2f(s[nt][e] - muse[r]);
        s[nt][e] = pv;
        l_run[r] += pv;
      }

    // O += P V  (fp16 operands: P keeps 11 mantissa bits)
#pragma unroll
    for (int kk = 0; kk < kKT / 16; ++kk) {
      uint32_t pf[4];
      pf[0] = pack2_f32<__half>(s[2 * kk][0], s[2 * kk][1]);
      pf[1] = pack2_f32<__half>(s[2 * kk][2], s[2 * kk][3]);
      pf[2] = pack2_f32<__half>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pf[3] = pack2_f32<__half>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int j = 0; j < D / 16; ++j) {
        uint32_t b0, b1, b2, b3;
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = j * 2 + (lane >> 4);
        ldmatrix_x4_trans(smem_u32(sV + key * D + ((ch ^ (key & 7)) * 8)), b0, b1, b2, b3);
        Mma<__half>::run(o[2 * j], pf, b0, b1);
        Mma<__half>::run(o[2 * j + 1], pf, b2, b3);
      }
    }
  }

  // epilogue: normalise, write final rows (single split) or split partials
  const bool single = (S == 1);
  const int pslot = single ? 0 : (p.part_begin[ri] + local);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_run[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int row = warp * 16 + (lane >> 2) + 8 * r;
    if (row >= nrows) continue;
    const float den = (l > 0.0f || l != l) ? l : 1.0f;
    const float inv = 1.0f / den;
    const float lse = (m_run[r] + log2f(den)) * 0.69314718055994531f;
    float* dst;
    float* lse_dst;
    if (single) {
      const int tl = row / G, hg = row - (row / G) * G;
      const int64_t qrow = (int64_t)(q_start + tok0 + tl) * a.hq + (int64_t)h * G + hg;
      dst = a.out + qrow * D;
      lse_dst = a.lse + qrow;
    } else {
      const int64_t prow = ((int64_t)pslot * a.hk + h) * ROWS + row;
      dst = a.part_o + prow * D;
      lse_dst = a.part_lse + prow;
    }
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt) {
      const int col = nt * 8 + 2 * (lane & 3);
      *reinterpret_cast<float2*>(dst + col) = make_float2(o[nt][2 * r] * inv, o[nt][2 * r + 1] * inv);
    }
    if ((lane & 3) == 0) *lse_dst = lse;
  }
}

// Combine split-KV partials of one row (requests with splits > 1).  Joint
// form of the pairwise merge of slab_attention.py:156-194: -inf partials get
// weight 0, NaN propagates, an all-empty row yields O = 0, LSE = -inf.
template <int D>
__global__ void split_combine_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p) {
  const int mrow = blockIdx.x, h = blockIdx.y;
  const int ROWS = p.rows;
  const int ri = find_bucket(p.merge_begin, p.num_req, mrow / ROWS) ;
  const int local = mrow - p.merge_begin[ri] * ROWS;
  const int qb = local / ROWS, row = local - (local / ROWS) * ROWS;
  const int S = p.splits[ri];
  const int nqb = (p.item_begin[ri + 1] - p.item_begin[ri]) / S;
  const int G = a.group;
  const int tok0 = qb * p.tpb;
  const int ntok = min(p.tpb, p.q_len[ri] - tok0);
  if (row >= ntok * G) return;
  const int first_local = (nqb - 1 - qb) * S;
  const int64_t pbase = p.part_begin[ri] + first_local;
  float m = -INFINITY;
  for (int sp = 0; sp < S; ++sp) m = nan_max(m, a.part_lse[((pbase + sp) * a.hk + h) * ROWS + row]);
  const float msafe = (m == -INFINITY) ? 0.0f : m;
  const int d0 = threadIdx.x * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.0f;
  for (int sp = 0; sp < S; ++sp) {
    const int64_t prow = ((pbase + sp) * a.hk + h) * ROWS + row;
    const float l = a.part_lse[prow];
    const float w = (l == -INFINITY) ? 0.0f : expf(l - msafe);
    wsum += w;
    if (w != 0.0f) {
      const float4 v = *reinterpret_cast<const float4*>(a.part_o + prow * D + d0);
      acc.x += w * v.x; acc.y += w * v.y; acc.z += w * v.z; acc.w += w * v.w;
    }
  }
  const float den = (wsum == 0.0f) ? 1.0f : wsum;
  const int tl = row / G, hg = row - (row / G) * G;
  const int64_t qrow = (int64_t)(p.q_start[ri] + tok0 + tl) * a.hq + (int64_t)h * G + hg;
  *reinterpret_cast<float4*>(a.out + qrow * D + d0) =
      make_float4(acc.x / den, acc.y / den, acc.z / den, acc.w / den);
  if (threadIdx.x == 0) a.lse[qrow] = m + logf(den);
}

// K4: kernels/slab_attention.py:156-194 (_merge_slab), one warp per (row, head).
template <typename P>
OSCAR_DEVINL float part_at(const P* p, int64_t i);
template <> OSCAR_DEVINL float part_at<float>(const float* p, int64_t i) { return p[i]; }
template <> OSCAR_DEVINL float part_at<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <> OSCAR_DEVINL float part_at<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }

template <typename P>
__global__ void merge_slab_kernel(float* __restrict__ out, float* __restrict__ lse, int64_t out_rows,
                                  const P* __restrict__ part,
                                  const float* __restrict__ part_lse, int64_t n, int hq, int d, int64_t start,
                                  const int32_t* __restrict__ ids) {
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= n * hq) return;
  const int64_t i = w / hq;
  const int head = (int)(w - i * hq);
  const int64_t tq = (ids != nullptr) ? (int64_t)ids[i] : start + i;
  if (tq < 0 || tq >= out_rows) {
    if (lane == 0) flag_error(8u);
    return;
  }
  const int64_t target = tq * hq + head;
  const float old_lse = lse[target];
  const float new_lse = part_lse[w];
  const float maximum = nan_max(old_lse, new_lse);
  const float safe = (maximum == -INFINITY) ? 0.0f : maximum;
  const float alpha = expf(old_lse - safe);
  const float beta = expf(new_lse - safe);
  float denom = alpha + beta;
  denom = (denom == 0.0f) ? 1.0f : denom;
  const bool old_empty = (old_lse == -INFINITY), new_empty = (new_lse == -INFINITY);
  for (int c = lane; c < d; c += 32) {
    const float ov = old_empty ? 0.0f : out[target * d + c];
    const float nv = new_empty ? 0.0f : part_at<P>(part, w * d + c);
    out[target * d + c] = (ov * alpha + nv * beta) / denom;
  }
  if (lane == 0) lse[target] = maximum + logf(denom);
}

}  // namespace oscar
