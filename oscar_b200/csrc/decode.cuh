// Decode / MTP attention over paged INT2 history: the GQA-shared streaming kernel.
//
// One CTA = 4 warps = one (request, kv head, history split).  All T x G query
// rows of the request's GQA group (<= 24 rows, NT n-tiles of 8) share every
// history token, which is read once from HBM as packed bytes -- K slot bytes
// [0:96) (fp16 K/V scale+zero, pad, 64 B K codes), V slot bytes [0:64) and the
// token's staging owner tag -- through a 4-stage cp.async ring of 64-token
// stages.  Nothing is dequantized to memory: the codes become mma.sync
// operands in registers.
//
// Values follow the reference's rounding chain exactly,
// T(fp16(code * scale + zero)) for history and T(fp16(x)) for staged fp32
// (streaming_attention.py:116-124), T being the query dtype.  A token's four
// possible values are a PRMT look-up table (X = low bytes, Y = high bytes);
// the tables of a stage's 64 tokens are built once, cooperatively.
//
// S^T = K Q^T (tokens x rows, query dtype): thread t of a quad owns dims
// [64t, 64t+64) of its two tokens; k-chunk c pairs dims 64t+4c+{0,1} and
// 64t+4c+{2,3}; the Q^T fragments (registers, loaded once) follow the same
// permutation.  Staged tokens (owner hits) are masked here: staged_item
// attends them from their fp32 staging rows and writes a separate partial.
//
// O^T = V^T P^T (dims x rows, fp16): PRMT selects same-token value pairs and
// a second PRMT transposes two tokens' pairs into each A register (k runs over
// tokens).  The V table holds fp16 bit patterns of the chain's values, exact
// because those values passed through fp16; P is fp16 (11-bit mantissa).
// Warp w owns V-code bytes [16w, 16w+16): m-tile e holds code e of bytes
// 16w+2g (rows g) and 16w+2g+1 (rows g+8).
//
// Only history positions [0, prefix) are processed here; the causal current
// chunk and the merge of all partials run in decode_combine_kernel.
#pragma once

#include "attention.cuh"

namespace oscar {

constexpr int kDecStage = 64;
constexpr int kDecNS = 4;
constexpr int kDecKBytes = 96;
constexpr int kDecVBytes = 64;
constexpr int kDecMaxPages = 512;
constexpr int kDecPStride = 72;  // halves per P row (64 + 8 pad: conflict-free B loads)

struct DecSmem {
  uint8_t k[kDecNS][kDecStage][kDecKBytes];
  uint8_t v[kDecNS][kDecStage][kDecVBytes];
  long long own[kDecNS][kDecStage];
  int btab[kDecMaxPages];
  __half pv[24][kDecPStride];  // P (fp16), [row][token]
  uint2 klut[kDecStage];       // K values (query dtype): X = low bytes, Y = high bytes
  uint2 vlut[kDecStage];       // V values (fp16 bit patterns)
  float red[4][24];
  float lred[4][24];
  unsigned int hits[2];
};

OSCAR_DEVINL void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
OSCAR_DEVINL void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
OSCAR_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
OSCAR_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

OSCAR_DEVINL uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// The 16 codes of a word -> 8 PRMT selectors, one per consecutive code pair
// (2k, 2k+1); a pair's selector nibbles are [ca, ca+4, cb, cb+4] so that
// PRMT(X, Y, sel) yields the two 16-bit values (low half = code 2k).
OSCAR_DEVINL void pair_selectors(uint32_t w, uint32_t (&sel)[8]) {
  const uint32_t e = w & 0x33333333u;
  const uint32_t o = (w >> 2) & 0x33333333u;
  const uint32_t t0 = prmt(e, o, 0x5140u);  // [e.b0, o.b0, e.b1, o.b1]
  const uint32_t t1 = prmt(e, o, 0x7362u);  // [e.b2, o.b2, e.b3, o.b3]
  const uint32_t s0 = (t0 & 0x03030303u) * 0x11u + 0x40404040u;         // pairs 0 (lo), 2 (hi)
  const uint32_t s1 = ((t0 >> 4) & 0x03030303u) * 0x11u + 0x40404040u;  // pairs 1, 3
  const uint32_t s2 = (t1 & 0x03030303u) * 0x11u + 0x40404040u;         // pairs 4, 6
  const uint32_t s3 = ((t1 >> 4) & 0x03030303u) * 0x11u + 0x40404040u;  // pairs 5, 7
  sel[0] = s0;
  sel[1] = s1;
  sel[2] = s0 >> 16;
  sel[3] = s1 >> 16;
  sel[4] = s2;
  sel[5] = s3;
  sel[6] = s2 >> 16;
  sel[7] = s3 >> 16;
}

// value of the reference chain T(fp16(x)) ...
template <typename T>
OSCAR_DEVINL T chain(float x) {
  return Elem<T>::from_f16(__float2half_rn(x));
}
// ... and the same value as fp16 (exact: it came from fp16; bf16 can round
// 65504 up to 65536, which is clamped)
template <typename T>
OSCAR_DEVINL __half chain_f16(float x) {
  const float v = Elem<T>::to_f32(chain<T>(x));
  return __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f));
}

OSCAR_DEVINL uint2 lut_from(uint32_t p01, uint32_t p23) {
  return make_uint2(prmt(p01, p23, 0x6420u), prmt(p01, p23, 0x7531u));
}

template <typename T>
OSCAR_DEVINL uint2 make_klut(float s, float z) {
  T v[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) v[c] = chain<T>(__fadd_rn(__fmul_rn((float)c, s), z));
  return lut_from(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]));
}

template <typename T>
OSCAR_DEVINL uint2 make_vlut(float s, float z) {
  __half v[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) v[c] = chain_f16<T>(__fadd_rn(__fmul_rn((float)c, s), z));
  return lut_from(pack2<__half>(v[0], v[1]), pack2<__half>(v[2], v[3]));
}

// ---------------------------------------------------------------------------
// Staged tokens.  A history position is staged when its staging seat is owned
// by its block: owner[(blk % rows) * bs + off] == blk (backend.py:172-176);
// it then attends with T(fp16(x)) of its fp32 staging rows instead of its
// INT2 codes (streaming_attention.py:116-124).  The decode CTAs mask staged
// positions; one staged item per history split lists them in position order,
// gathers 16 at a time with cp.async (double-buffered) and writes its own
// normalised partial (O, LSE), or LSE = -inf when its split holds none.
constexpr int kStWin = 512;      // positions listed per window
constexpr int kStGroup = 16;     // staged tokens per MMA group
constexpr int kStKStride = 264;  // floats per staged K row (conflict-free A-fragment loads)
constexpr int kStVStride = 260;  // floats per staged V row

struct StagedSmem {
  float k[2][kStGroup][kStKStride];
  float v[2][kStGroup][kStVStride];
  int seat[kStWin];
  int pos[kStWin];
  float red[4][kStGroup][33];  // per-warp partial S^T [token][row]
  __half pt[32][24];           // P [row][token]
  float alpha[32];
  float lsum[32];
  float mrow[32];
  int wsum[4];
};

template <typename T, int NT>
OSCAR_DEVINL void staged_item(const AttnArgs& a, const AttnPlan& p, int item, uint8_t* smem_raw) {
  constexpr int D = 256;
  StagedSmem& sm = *reinterpret_cast<StagedSmem*>(smem_raw);
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ri = find_bucket(p.item_begin, p.num_req, item);
  const int sp = item - p.item_begin[ri];
  const int req = p.req_id[ri];
  const int q_start = p.q_start[ri], qlen = p.q_len[ri], seq = p.seq[ri], prefix = p.prefix[ri];
  const int G = a.group;
  const int R = qlen * G;
  const int lo = sp * p.chunk[ri];
  const int hi = min(lo + p.chunk[ri], prefix);
  const int bs = a.bs;
  const int rows_mod = (int)a.stage_rows;

  // Q^T fragments of this warp's dims [64w, 64w + 64): chunk c covers 64w + 16c + [0, 16)
  uint32_t qf[4][NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int row = 8 * nt + g;
    const bool ok = row < R;
    const T* qrow = reinterpret_cast<const T*>(a.q) +
                    ((int64_t)(q_start + (ok ? row / G : 0)) * a.hq + (int64_t)h * G + (ok ? row % G : 0)) * D;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int k0 = 64 * warp + 16 * c + 2 * t;
      qf[c][nt][0] = ok ? *reinterpret_cast<const uint32_t*>(qrow + k0) : 0u;
      qf[c][nt][1] = ok ? *reinterpret_cast<const uint32_t*>(qrow + k0 + 8) : 0u;
    }
  }

  // softmax state: threads 4r .. 4r+3 own row r (tokens 4q .. 4q+3 of a group)
  const int srow = tid >> 2, sq = tid & 3;
  const bool srow_ok = srow < 8 * NT;
  const int slim = (srow < R) ? seq - qlen + srow / G + 1 : -1;  // visible positions are < slim
  float m_r = -INFINITY, l_r = 0.0f;
  float o[4][NT][4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[e][nt][0] = o[e][nt][1] = o[e][nt][2] = o[e][nt][3] = 0.0f;

  for (int w0 = lo; w0 < hi; w0 += kStWin) {
    __syncthreads();  // the previous window's list is consumed
    // ---- list the staged positions of [w0, w0 + kStWin), 4 consecutive ones per thread
    int seats[4];
    bool hit[4];
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int pos = w0 + 4 * tid + j;
      hit[j] = false;
      seats[j] = 0;
      if (pos < hi) {
        const int pg = pos / bs, off = pos - pg * bs;
        const int blk = a.bt[(int64_t)req * a.bt_stride + pg];
        if (blk < 0 || blk >= a.num_blocks) {
          flag_error(2u);
        } else {
          seats[j] = (blk % rows_mod) * bs + off;
          hit[j] = a.owner[seats[j]] == (int64_t)blk;
        }
      }
      cnt += hit[j] ? 1 : 0;
    }
    int incl = cnt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    if (lane == 31) sm.wsum[warp] = incl;
    __syncthreads();
    int wbase = 0, total = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      wbase += (w < warp) ? sm.wsum[w] : 0;
      total += sm.wsum[w];
    }
    int at = wbase + incl - cnt;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (hit[j]) {
        sm.seat[at] = seats[j];
        sm.pos[at] = w0 + 4 * tid + j;
        ++at;
      }
    __syncthreads();

    // ---- groups of 16 staged tokens
    const int ng = (total + kStGroup - 1) / kStGroup;
    auto issue = [&](int gi) {
      if (gi < ng) {
        const int buf = gi & 1;
#pragma unroll 4
        for (int tok = 0; tok < kStGroup; ++tok) {
          const int li = gi * kStGroup + tok;
          if (li < total) {
            const int64_t rowoff = ((int64_t)sm.seat[li] * a.hk + h) * D;
            if (tid < 64)
              cp_async16(&sm.k[buf][tok][tid * 4], a.stage_k + rowoff + tid * 4);
            else
              cp_async16(&sm.v[buf][tok][(tid - 64) * 4], a.stage_v + rowoff + (tid - 64) * 4);
          } else if (tid >= 64) {
            *reinterpret_cast<float4*>(&sm.v[buf][tok][(tid - 64) * 4]) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      cp_async_commit();
    };
    issue(0);
    for (int gi = 0; gi < ng; ++gi) {
      issue(gi + 1);
      cp_async_wait<1>();
      __syncthreads();
      const int buf = gi & 1;

      // partial S^T = K Q^T over this warp's 64 dims
      float sacc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int k0 = 64 * warp + 16 * c + 2 * t;
        const float2 f0 = *reinterpret_cast<const float2*>(&sm.k[buf][g][k0]);
        const float2 f1 = *reinterpret_cast<const float2*>(&sm.k[buf][g + 8][k0]);
        const float2 f2 = *reinterpret_cast<const float2*>(&sm.k[buf][g][k0 + 8]);
        const float2 f3 = *reinterpret_cast<const float2*>(&sm.k[buf][g + 8][k0 + 8]);
        const uint32_t af[4] = {pack2<T>(chain<T>(f0.x), chain<T>(f0.y)), pack2<T>(chain<T>(f1.x), chain<T>(f1.y)),
                                pack2<T>(chain<T>(f2.x), chain<T>(f2.y)), pack2<T>(chain<T>(f3.x), chain<T>(f3.y))};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<T>::run(sacc[nt], af, qf[c][nt][0], qf[c][nt][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sm.red[warp][g][8 * nt + 2 * t] = sacc[nt][0];
        sm.red[warp][g][8 * nt + 2 * t + 1] = sacc[nt][1];
        sm.red[warp][g + 8][8 * nt + 2 * t] = sacc[nt][2];
        sm.red[warp][g + 8][8 * nt + 2 * t + 1] = sacc[nt][3];
      }
      __syncthreads();

      // online softmax over the group, row srow, tokens 4sq .. 4sq+3
      if (srow_ok) {
        float x[4];
        float gm = -INFINITY;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int tok = 4 * sq + k, li = gi * kStGroup + tok;
          const float sv = sm.red[0][tok][srow] + sm.red[1][tok][srow] + sm.red[2][tok][srow] + sm.red[3][tok][srow];
          const bool valid = li < total && sm.pos[li] < slim;
          x[k] = valid ? sv * a.scale_log2 : -INFINITY;
          gm = fmaxf(gm, x[k]);
        }
        gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 1));
        gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 2));
        const float m_new = fmaxf(m_r, gm);
        const float muse = (m_new == -INFINITY) ? 0.0f : m_new;
        const float alpha = exp2f(m_r - muse);
        float ps = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float pk = exp2f(x[k] - muse);
          ps += pk;
          sm.pt[srow][4 * sq + k] = __float2half_rn(pk);
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        l_r = l_r * alpha + ps;
        m_r = m_new;
        if (sq == 0) sm.alpha[srow] = alpha;
      }
      __syncthreads();

      // O^T += V^T P^T for this warp's dims 64w + 16e + [0, 16)
      uint32_t bfr[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float a0 = sm.alpha[8 * nt + 2 * t], a1 = sm.alpha[8 * nt + 2 * t + 1];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o[e][nt][0] *= a0;
          o[e][nt][1] *= a1;
          o[e][nt][2] *= a0;
          o[e][nt][3] *= a1;
        }
        bfr[nt][0] = *reinterpret_cast<const uint32_t*>(&sm.pt[8 * nt + g][2 * t]);
        bfr[nt][1] = *reinterpret_cast<const uint32_t*>(&sm.pt[8 * nt + g][2 * t + 8]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d0 = 64 * warp + 16 * e + g;
        const float(*vb)[kStVStride] = sm.v[buf];
        const uint32_t af[4] = {
            pack2<__half>(chain_f16<T>(vb[2 * t][d0]), chain_f16<T>(vb[2 * t + 1][d0])),
            pack2<__half>(chain_f16<T>(vb[2 * t][d0 + 8]), chain_f16<T>(vb[2 * t + 1][d0 + 8])),
            pack2<__half>(chain_f16<T>(vb[2 * t + 8][d0]), chain_f16<T>(vb[2 * t + 9][d0])),
            pack2<__half>(chain_f16<T>(vb[2 * t + 8][d0 + 8]), chain_f16<T>(vb[2 * t + 9][d0 + 8]))};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<__half>::run(o[e][nt], af, bfr[nt][0], bfr[nt][1]);
      }
      __syncthreads();  // buffers, red and pt are rewritten by the next group
    }
    cp_async_wait<0>();
  }

  // ---- epilogue: the staged partial of this split
  __syncthreads();
  if (srow_ok && sq == 0) {
    sm.lsum[srow] = l_r;
    sm.mrow[srow] = m_r;
  }
  __syncthreads();
  const int64_t pslot = (int64_t)p.total_items + p.part_begin[ri] + sp;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int row = 8 * nt + 2 * t + j;
      if (row >= R) continue;
      const float l = sm.lsum[row];
      if (!(l > 0.0f) && l == l) continue;  // no staged token: the combine skips this O
      const float inv = 1.0f / l;
      float* dst = a.part_o + ((pslot * a.hk + h) * (NT * 8) + row) * D;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dst[64 * warp + 16 * e + g] = o[e][nt][j] * inv;
        dst[64 * warp + 16 * e + g + 8] = o[e][nt][2 + j] * inv;
      }
    }
  if (tid < R) {
    const float l = sm.lsum[tid];
    a.part_lse[(pslot * a.hk + h) * (NT * 8) + tid] =
        (l > 0.0f || l != l) ? (sm.mrow[tid] + log2f(l)) * 0.69314718055994531f : -INFINITY;
  }
}

template <typename T, int NT>
__global__ void __launch_bounds__(128, 2)
    decode_attn_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p, int staged_items) {
  constexpr int D = 256;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the first staged_items CTAs attend the staged tokens of each split
  if ((int)blockIdx.x < staged_items) {
    staged_item<T, NT>(a, p, blockIdx.x, smem_raw);
    return;
  }
  DecSmem& sm = *reinterpret_cast<DecSmem*>(smem_raw);

  const int item = blockIdx.x - staged_items, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ri = find_bucket(p.item_begin, p.num_req, item);
  const int sp = item - p.item_begin[ri];
  const int req = p.req_id[ri];
  const int q_start = p.q_start[ri], qlen = p.q_len[ri], seq = p.seq[ri], prefix = p.prefix[ri];
  const int G = a.group;
  const int R = qlen * G;
  const int lo = sp * p.chunk[ri];
  const int hi = min(lo + p.chunk[ri], prefix);
  const int bs = a.bs;

  // ---- block-table slice of this split (bounds-checked)
  const int page0 = lo / bs;
  const int npages = (hi > lo) ? (hi - 1) / bs - page0 + 1 : 0;
  for (int i = tid; i < npages; i += 128) {
    int blk = a.bt[(int64_t)req * a.bt_stride + page0 + i];
    if (blk < 0 || blk >= a.num_blocks) {
      flag_error(2u);
      blk = 0;
    }
    sm.btab[i] = blk;
  }
  __syncthreads();

  const int nstages = (hi > lo) ? (hi - lo + kDecStage - 1) / kDecStage : 0;
  auto issue = [&](int st) {
    if (st < nstages) {
      const int slot = st % kDecNS;
      const int base = lo + st * kDecStage;
      for (int task = tid; task < kDecStage * 11; task += 128) {
        const int tok = task / 11, part = task - tok * 11;
        const int pos = base + tok;
        if (pos < hi) {
          const int pg = pos / bs, off = pos - pg * bs;
          const int64_t blk = sm.btab[pg - page0];
          if (part < 6) {
            cp_async16(&sm.k[slot][tok][part * 16], a.kc + blk * a.ksb + off * a.kst + (int64_t)h * a.ksh + part * 16);
          } else if (part < 10) {
            cp_async16(&sm.v[slot][tok][(part - 6) * 16],
                       a.vc + blk * a.vsb + off * a.vst + (int64_t)h * a.vsh + (part - 6) * 16);
          } else if (a.owner != nullptr) {
            cp_async8(&sm.own[slot][tok], a.owner + (blk % a.stage_rows) * bs + off);
          } else {
            sm.own[slot][tok] = -2;
          }
        } else if (part == 10) {
          sm.own[slot][tok] = -2;
        }
      }
    }
    cp_async_commit();
  };

  // ---- Q^T fragments: chunk c, n-tile nt -> row 8nt+g, dims 64t+4c..64t+4c+3
  uint32_t qf[16][NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int row = 8 * nt + g;
    const bool ok = row < R;
    const T* qrow = reinterpret_cast<const T*>(a.q) +
                    ((int64_t)(q_start + (ok ? row / G : 0)) * a.hq + (int64_t)h * G + (ok ? row % G : 0)) * D;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint2 v = make_uint2(0, 0);
      if (ok) v = *reinterpret_cast<const uint2*>(qrow + 64 * t + 4 * c);
      qf[c][nt][0] = v.x;
      qf[c][nt][1] = v.y;
    }
  }

  // C-fragment rows of this thread: 8nt + 2t + {0,1}, with their causal limits
  int lim[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int row = 8 * nt + 2 * t + j;
      lim[nt][j] = (row < R) ? min(hi, seq - qlen + row / G + 1) : -1;
    }

  float o[4][NT][4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[e][nt][0] = o[e][nt][1] = o[e][nt][2] = o[e][nt][3] = 0.0f;
  float m_run[NT][2], l_run[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      m_run[nt][j] = -INFINITY;
      l_run[nt][j] = 0.0f;
    }

#pragma unroll
  for (int s = 0; s < kDecNS - 1; ++s) issue(s);

  for (int st = 0; st < nstages; ++st) {
    cp_async_wait<kDecNS - 2>();
    __syncthreads();
    issue(st + kDecNS - 1);
    const int slot = st % kDecNS;
    const int base = lo + st * kDecStage;

    // ---------------- per-token value tables; staged tokens (owner hits) and
    // positions past the split get zero tables, and a bitmask marks the live ones
    {
      const int tok = tid >> 1, side = tid & 1;
      const uint8_t* mt = sm.k[slot][tok] + 4 * side;
      const int pos = base + tok;
      bool live = pos < hi;
      if (live) {
        const long long ow = sm.own[slot][tok];
        live = !(ow >= 0 && ow == (long long)sm.btab[pos / bs - page0]);
      }
      uint2 lut = make_uint2(0, 0);
      if (live) {
        const float sc = f16_bits_to_f32(ld_u16(mt)), zr = f16_bits_to_f32(ld_u16(mt + 2));
        lut = side ? make_vlut<T>(sc, zr) : make_klut<T>(sc, zr);
      }
      if (side) sm.vlut[tok] = lut; else sm.klut[tok] = lut;
      // lanes 2i and 2i+1 of a warp share token 16w + i
      const unsigned int b = __ballot_sync(0xffffffffu, live) & 0x55555555u;
      if (lane == 0) {
        unsigned int m16 = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) m16 |= ((b >> (2 * i)) & 1u) << i;
        reinterpret_cast<unsigned short*>(sm.hits)[warp] = (unsigned short)m16;
      }
    }
    __syncthreads();
    const unsigned int hm0 = sm.hits[0], hm1 = sm.hits[1];

    // ---------------- S^T = K Q^T for this warp's 16 tokens
    const int tk0 = warp * 16 + g, tk1 = tk0 + 8;
    float sacc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
    {
      const uint2 l0 = sm.klut[tk0], l1 = sm.klut[tk1];
      const uint4 w0 = *reinterpret_cast<const uint4*>(sm.k[slot][tk0] + 32 + 16 * t);
      const uint4 w1 = *reinterpret_cast<const uint4*>(sm.k[slot][tk1] + 32 + 16 * t);
      const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w};
      const uint32_t wb[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t sa[8], sb[8];
        pair_selectors(wa[i], sa);
        pair_selectors(wb[i], sb);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = 4 * i + cc;
          uint32_t af[4];
          af[0] = prmt(l0.x, l0.y, sa[2 * cc]);
          af[2] = prmt(l0.x, l0.y, sa[2 * cc + 1]);
          af[1] = prmt(l1.x, l1.y, sb[2 * cc]);
          af[3] = prmt(l1.x, l1.y, sb[2 * cc + 1]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Mma<T>::run(sacc[nt], af, qf[c][nt][0], qf[c][nt][1]);
        }
      }
    }

    // ---------------- mask, stage row max over the 4 warps, probabilities
    const unsigned int hword = (warp < 2) ? hm0 : hm1;
    const bool live0 = (hword >> (tk0 & 31)) & 1u, live1 = (hword >> (tk1 & 31)) & 1u;
    float mx[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float v0 = (live0 && base + tk0 < lim[nt][j]) ? sacc[nt][j] * a.scale_log2 : -INFINITY;
        const float v1 = (live1 && base + tk1 < lim[nt][j]) ? sacc[nt][2 + j] * a.scale_log2 : -INFINITY;
        sacc[nt][j] = v0;
        sacc[nt][2 + j] = v1;
        float m = fmaxf(v0, v1);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        mx[nt][j] = m;
      }
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) sm.red[warp][8 * nt + 2 * t + j] = mx[nt][j];
    }
    __syncthreads();
    float alpha[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int row = 8 * nt + 2 * t + j;
        const float smax = fmaxf(fmaxf(sm.red[0][row], sm.red[1][row]), fmaxf(sm.red[2][row], sm.red[3][row]));
        const float m_new = fmaxf(m_run[nt][j], smax);
        const float muse = (m_new == -INFINITY) ? 0.0f : m_new;
        alpha[nt][j] = exp2f(m_run[nt][j] - muse);
        m_run[nt][j] = m_new;
        const float p0 = exp2f(sacc[nt][j] - muse);
        const float p1 = exp2f(sacc[nt][2 + j] - muse);
        l_run[nt][j] = l_run[nt][j] * alpha[nt][j] + p0 + p1;
        sm.pv[row][tk0] = __float2half_rn(p0);
        sm.pv[row][tk1] = __float2half_rn(p1);
      }
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        o[e][nt][0] *= alpha[nt][0];
        o[e][nt][1] *= alpha[nt][1];
        o[e][nt][2] *= alpha[nt][0];
        o[e][nt][3] *= alpha[nt][1];
      }
    __syncthreads();

    // ---------------- O^T += V^T P^T (warp w: V-code bytes [16w, 16w+16))
    const uint8_t* vbase = &sm.v[slot][0][16 * warp + 2 * g];
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const int j0 = 16 * kc + 2 * t;
      // rv[token][k]: k = 0,1 -> codes (0,1),(2,3) of byte 16w+2g; k = 2,3 -> of byte 16w+2g+1
      uint32_t rv[4][4];
#pragma unroll
      for (int hp = 0; hp < 2; ++hp) {
        const int ja = j0 + 8 * hp, jb = ja + 1;
        const uint32_t w = ld_u16(vbase + ja * kDecVBytes) | (ld_u16(vbase + jb * kDecVBytes) << 16);
        uint32_t sel[8];
        pair_selectors(w, sel);
        const uint2 la = sm.vlut[ja], lb = sm.vlut[jb];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          rv[2 * hp][k] = prmt(la.x, la.y, sel[k]);
          rv[2 * hp + 1][k] = prmt(lb.x, lb.y, sel[4 + k]);
        }
      }
      uint32_t bfr[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const __half* prow = &sm.pv[8 * nt + g][0];
        bfr[nt][0] = *reinterpret_cast<const uint32_t*>(prow + j0);
        bfr[nt][1] = *reinterpret_cast<const uint32_t*>(prow + j0 + 8);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t tsel = (e & 1) ? 0x7632u : 0x5410u;
        uint32_t af[4];
        af[0] = prmt(rv[0][e >> 1], rv[1][e >> 1], tsel);            // dim of byte 16w+2g, tokens j0, j0+1
        af[1] = prmt(rv[0][2 + (e >> 1)], rv[1][2 + (e >> 1)], tsel);  // dim of byte 16w+2g+1
        af[2] = prmt(rv[2][e >> 1], rv[3][e >> 1], tsel);            // tokens j0+8, j0+9
        af[3] = prmt(rv[2][2 + (e >> 1)], rv[3][2 + (e >> 1)], tsel);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<__half>::run(o[e][nt], af, bfr[nt][0], bfr[nt][1]);
      }
    }
  }
  cp_async_wait<0>();

  // ---------------- epilogue: l over the 8 g-lanes and 4 warps, normalised partial
  __syncthreads();
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float l = l_run[nt][j];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      if (g == 0) sm.lred[warp][8 * nt + 2 * t + j] = l;
    }
  __syncthreads();
  const int pslot = p.part_begin[ri] + sp;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int row = 8 * nt + 2 * t + j;
      if (row >= R) continue;
      const float l = sm.lred[0][row] + sm.lred[1][row] + sm.lred[2][row] + sm.lred[3][row];
      const float den = (l > 0.0f || l != l) ? l : 1.0f;
      const float inv = 1.0f / den;
      const int64_t prow = ((int64_t)pslot * a.hk + h) * (NT * 8) + row;
      float* dst = a.part_o + prow * D;
      const float4 lo4 = make_float4(o[0][nt][j] * inv, o[1][nt][j] * inv, o[2][nt][j] * inv, o[3][nt][j] * inv);
      const float4 hi4 =
          make_float4(o[0][nt][2 + j] * inv, o[1][nt][2 + j] * inv, o[2][nt][2 + j] * inv, o[3][nt][2 + j] * inv);
      *reinterpret_cast<float4*>(dst + 4 * (16 * warp + 2 * g)) = lo4;
      *reinterpret_cast<float4*>(dst + 4 * (16 * warp + 2 * g + 1)) = hi4;
      if (warp == 0 && g == 0) a.part_lse[prow] = (m_run[nt][j] + log2f(den)) * 0.69314718055994531f;
    }
}

// Merge every partial of one query row -- the history splits, the staged
// partials and the causal current chunk (k_new/v_new keys 0 .. tl) -- with
// one thread per dim.  Final rows go to out/lse.
template <typename T>
__global__ void __launch_bounds__(256) decode_combine_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p,
                                                             int rows_stride, int staged) {
  constexpr int D = 256;
  __shared__ float wsh[256];
  __shared__ int64_t rsh[256];
  __shared__ int wcnt[8];
  __shared__ float ksc[32];
  __shared__ float red[8];
  const int ri = blockIdx.x;
  const int h = blockIdx.y / rows_stride, row = blockIdx.y - (blockIdx.y / rows_stride) * rows_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q_start = p.q_start[ri], qlen = p.q_len[ri], seq = p.seq[ri], prefix = p.prefix[ri];
  const int G = a.group;
  if (row >= qlen * G) return;
  const int tl = row / G, hg = row - tl * G;
  const int64_t qrow = (int64_t)(q_start + tl) * a.hq + (int64_t)h * G + hg;
  const int S = p.splits[ri];
  const int np = (prefix > 0) ? S * (staged ? 2 : 1) : 0;
  const int64_t pbase = p.part_begin[ri];
  auto prow_of = [&](int i) -> int64_t {
    const int64_t slot = (i < S) ? pbase + i : (int64_t)p.total_items + pbase + (i - S);
    return (slot * a.hk + h) * rows_stride + row;
  };
  const int nkeys = (a.k_new != nullptr) ? min(seq - prefix - (qlen - 1 - tl), 32) : 0;

  // current-chunk scores (natural-log units), one warp per key
  for (int j = warp; j < nkeys; j += 8) {
    const uint4 qu = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.q) + qrow * D + 8 * lane);
    const uint4 ku = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.k_new) +
                                                     ((int64_t)(q_start + j) * a.hk + h) * D + 8 * lane);
    const T* qe = reinterpret_cast<const T*>(&qu);
    const T* ke = reinterpret_cast<const T*>(&ku);
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) d = fmaf(Elem<T>::to_f32(qe[i]), Elem<T>::to_f32(ke[i]), d);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o2);
    if (lane == 0) ksc[j] = d * a.scale_log2 * 0.69314718055994531f;
  }
  // global max over partial LSEs and key scores (NaN propagates)
  float mx = -INFINITY;
  for (int i = tid; i < np; i += 256) mx = nan_max(mx, a.part_lse[prow_of(i)]);
  __syncthreads();
  if (tid < nkeys) mx = nan_max(mx, ksc[tid]);
#pragma unroll
  for (int o2 = 16; o2 > 0; o2 >>= 1) mx = nan_max(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  float M = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) M = nan_max(M, red[w]);
  const float Mu = (M == -INFINITY) ? 0.0f : M;

  // weights of the non-empty partials, compacted in order, then a weighted
  // sum with independent loads (empty staged partials hold no O)
  float acc = 0.0f, L = 0.0f;
  for (int i0 = 0; i0 < np; i0 += 256) {
    const int i = i0 + tid;
    float w = 0.0f;
    int64_t prow = 0;
    if (i < np) {
      prow = prow_of(i);
      const float ls = a.part_lse[prow];
      w = (ls == -INFINITY) ? 0.0f : expf(ls - Mu);
    }
    const bool keep = w != 0.0f;
    const unsigned int bal = __ballot_sync(0xffffffffu, keep);
    __syncthreads();  // the previous batch's list is consumed
    if (lane == 0) wcnt[warp] = __popc(bal);
    __syncthreads();
    int at = 0, cnt = 0;
#pragma unroll
    for (int w2 = 0; w2 < 8; ++w2) {
      at += (w2 < warp) ? wcnt[w2] : 0;
      cnt += wcnt[w2];
    }
    if (keep) {
      const int k = at + __popc(bal & ((1u << lane) - 1u));
      wsh[k] = w;
      rsh[k] = prow;
    }
    __syncthreads();
    int k = 0;
    for (; k + 4 <= cnt; k += 4) {
      const float x0 = a.part_o[rsh[k] * D + tid], x1 = a.part_o[rsh[k + 1] * D + tid];
      const float x2 = a.part_o[rsh[k + 2] * D + tid], x3 = a.part_o[rsh[k + 3] * D + tid];
      acc = fmaf(wsh[k], x0, acc);
      acc = fmaf(wsh[k + 1], x1, acc);
      acc = fmaf(wsh[k + 2], x2, acc);
      acc = fmaf(wsh[k + 3], x3, acc);
      L += wsh[k];
      L += wsh[k + 1];
      L += wsh[k + 2];
      L += wsh[k + 3];
    }
    for (; k < cnt; ++k) {
      acc = fmaf(wsh[k], a.part_o[rsh[k] * D + tid], acc);
      L += wsh[k];
    }
  }
  for (int j = 0; j < nkeys; ++j) {
    const float w = expf(ksc[j] - Mu);
    const T v = reinterpret_cast<const T*>(a.v_new)[((int64_t)(q_start + j) * a.hk + h) * D + tid];
    acc = fmaf(w, Elem<T>::to_f32(v), acc);
    L += w;
  }
  const float den = (L > 0.0f || L != L) ? L : 1.0f;
  a.out[qrow * D + tid] = acc / den;
  if (tid == 0) a.lse[qrow] = (M == -INFINITY) ? -INFINITY : Mu + logf(den);
}

}  // namespace oscar
