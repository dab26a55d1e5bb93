// Decode / MTP attention over paged INT2 history on the 5th-generation tensor
// cores: the tcgen05 + TMEM + TMA kernel.
//
// One CTA per SM = one (request, kv head, history split); 800 threads.
//   warp 24: TMA producer and MMA issuer, an event loop over its three queues
//     (QK, PV, TMA refills).  The split's INT2 history arrives in 128-token
//     stages through a 2-slot ring: K slot bytes [0:48) and [48:96), V slot
//     bytes [0:48) and [16:64) of every token, four 2D tensor-map boxes per
//     page whose 48-byte rows put the 8 tokens of a shared-memory wavefront on
//     8 distinct bank groups.
//   warps 0-15 (dequant): warp w serves tokens 32 (w % 4) .. + 31 (its TMEM
//     lane quarter) in role q = w / 4: K dims [0, 128), K dims [128, 256), V
//     dims [0, 128) or V dims [128, 256) of those tokens.
//   warps 16-23 (softmax): warp 16 + 4 hr + lq serves the tokens of lane
//     quarter lq for query rows [16 hr, 16 hr + 16).
//   Each role waits only on the buffers it touches; no barrier spans the CTA
//   inside a stage.
//
// Staging window (owner[(blk % rows) * bs + off] == blk, backend.py:172-176):
// staged positions inside the split's own range are masked in its INT2 stages
// (the owner tags of each stage's seats arrive by bulk copy with the stage).
// The request's staged positions are attended by the CTAs of the request in
// turn, 32-position group g by split g % splits, so that a sink or recent
// window spreads over many CTAs instead of loading one SM with its fp32 rows:
// the prologue scans this CTA's groups, and "staged stages" over their staged
// positions (128 per stage) run before the INT2 stages, their fp32 loads
// overlapping the TMA latency of the first INT2 stages.
//
// Per stage:
//   K -> values T(fp16(code * scale + zero)) (streaming_attention.py:116-124)
//     by PRMT look-up in the token's 4-entry table (staged: T(fp16(x))),
//     written into tensor memory as the A operand (lanes = tokens, K-major).
//     A 17th k-step carries a per-token bias, 0 or -inf for masked tokens
//     (whose K is zero), against a column of ones in Q: masking costs the
//     softmax nothing.
//   S^T = K Q^T: M = 128 tokens, N = 32 query rows, K = 256 dims (+16); Q sits
//     in shared memory (K-major, loaded once).
//   V -> fp16 values (the chain's values are fp16-exact) in a shared V^T tile
//     (MN-major: dims contiguous per token).
//   softmax: each thread loads its token's 16 scores from TMEM.  The running
//     row maximum moves only when a score exceeds it by more than 15 (log2
//     units): P = 2^(x - m) stays <= 2^15 in fp16, and O/l are rescaled on
//     those stages only.  P^T goes to shared memory (MN-major).
//   O^T += V^T P^T: two M = 128 dim halves, N = 32 rows, K = 16 tokens per
//     instruction, accumulated in TMEM across the split; L += 1 P^T beside it.
// The normalised partial (O in fp16, LSE) goes to the workspace;
// tc_combine_kernel merges the splits with the causal current chunk.
//
// Dim orders inside each 16-dim group: K columns (pairs of k elements) hold
// dims (0,2) (1,3) (4,6) (5,7) (8,10) (9,11) (12,14) (13,15), so that the four
// columns 2m, 2m + 1 of a token come from its dims 4m .. 4m + 3 (a 16-byte
// piece of an fp32 row: staged rows load 64 contiguous bytes per token); Q is
// loaded in the same order.  V's M index runs over dims [0,2,..,14,1,3,..,15]
// (the order the look-up emits them), mapped back when the partial is written.
#pragma once

#include <climits>
#include <cstddef>
#include <type_traits>

#include "decode.cuh"
#include "tc.cuh"

namespace oscar {

constexpr int kTcStage = 128;
constexpr int kTcDeqWarps = 16;  // dequant warps: K / V halves x TMEM lane quarters
constexpr int kTcSmWarps = 8;    // softmax warps: one per (TMEM lane quarter, 16-row half of the query rows)
constexpr int kTcQuarters = 4;   // TMEM lane quarters (a warp reaches lanes 32 (warp % 4) .. + 31)
constexpr int kTcProdWarp = kTcDeqWarps + kTcSmWarps;  // TMA producer and MMA issuer
constexpr int kTcThreads = 32 * (kTcProdWarp + 1);     // 800
constexpr int kTcCompute = 32 * kTcDeqWarps;
constexpr int kTcRows = 32;   // N of both MMAs: query rows (GQA group x MTP tokens)
constexpr int kTcK = 272;     // QK reduction: 256 dims + the bias k-step
// TMEM columns: A_K[0] [0,136) | ones [136,144) | S[0] [160,192) | S[1] [192,224) | O [224,288) |
// A_K[1] [288,424) | row sums L [448,480)
constexpr int kTcCols = 512;
constexpr int kTcColA0 = 0, kTcColOnes = 136, kTcColA1 = 288, kTcColS = 160, kTcColO = 224, kTcColL = 448;
constexpr int kTcMaxStages = 64;  // INT2 stages per split (staged bitmask capacity)
constexpr int kTcMaxWords = kTcMaxStages * kTcStage / 32;
constexpr int kTcMaxPages = kTcMaxStages * kTcStage / 8 + 2;
constexpr uint32_t kTcVtSbo = 2048;          // V^T / P^T: bytes between 8-element MN groups (16 token groups x 128 B)
constexpr uint32_t kTcQSbo = kTcK / 8 * 128;  // Q: bytes between 8-row groups (34 k-groups x 128 B)
constexpr float kTcHeadroom = 15.0f;

constexpr int kTcRow = 48;  // bytes per token row of each raw box

struct TcSmem {
  uint8_t ka[2][kTcStage][kTcRow];  // K slot bytes [0, 48): K/V scale+zero, pad, codes of dims 0..63
  uint8_t kb[2][kTcStage][kTcRow];  // K slot bytes [48, 96): codes of dims 64..255
  uint8_t va[2][kTcStage][kTcRow];  // V slot bytes [0, 48)
  uint8_t vb[2][kTcStage][kTcRow];  // V slot bytes [16, 64)
  uint8_t vt[2][256 * kTcStage * 2];      // V^T: address(tok, m) = (m/8)*2048 + (tok/8)*128 + (tok%8)*16 + (m%8)*2
  uint8_t pt[2][kTcRows * kTcStage * 2];  // P^T: address(tok, n) = (n/8)*2048 + (tok/8)*128 + (tok%8)*16 + (n%8)*2
  uint8_t qb[kTcRows * kTcK * 2];      // Q:   address(n, k)   = (n/8)*4352 + (k/8)*128 + (n%8)*16 + (k%8)*2
  int btab[kTcMaxPages];
  alignas(16) int64_t own[2][kTcStage];  // owner tags of the stage's seats (bulk-copied with the stage)
  uint32_t gmask[kTcMaxWords];  // staged positions this CTA attends: 32-position group sp + k * splits
  int gpref[kTcMaxWords + 1];   // exclusive prefix counts of gmask
  int64_t srow[kTcStage];       // first staged stage: fp32 row offset per token slot (-1: none)
  int spos[kTcStage];           // first staged stage: position per token slot
  int lim[kTcRows];             // cache-only chunks: row r sees positions < lim[r]
  alignas(16) int red[kTcQuarters][kTcRows];    // slow-path row maxima of the softmax warps ([quarter][row])
  alignas(16) float mrow[kTcQuarters][kTcRows];  // running row maxima (log2 units), a copy per softmax warp
  // per buffer (a barrier that could complete twice before its waiter looks
  // would be read as not complete by a parity wait)
  unsigned long long bar_full[2], bar_empty[2], bar_k[2], bar_s[2], bar_v[2], bar_p[2], bar_pv[2];
  uint32_t tmem;
  int abort;
  int n_staged;
};
// vector accesses (uint4) and TMA destinations rely on these
static_assert(offsetof(TcSmem, kb) % 128 == 0 && offsetof(TcSmem, va) % 128 == 0 &&
                  offsetof(TcSmem, vb) % 128 == 0 && offsetof(TcSmem, vt) % 16 == 0 && offsetof(TcSmem, pt) % 16 == 0 &&
                  offsetof(TcSmem, qb) % 16 == 0 && sizeof(TcSmem) <= 227 * 1024,
              "TcSmem layout");

// dim of the M/K index m (16-dim groups emitted as [0,2,..,14,1,3,..,15])
OSCAR_DEVINL int tc_dim(int m) { return (m & ~15) | ((m & 7) << 1) | ((m >> 3) & 1); }

// one word of 16 codes -> 8 registers of 2 values each, in the permuted order:
// registers (0..3) hold dims (0,2) (4,6) (8,10) (12,14), (4..7) dims (1,3) .. (13,15)
OSCAR_DEVINL void tc_lut_word(uint32_t w, uint32_t x, uint32_t y, uint32_t* r) {
  const uint32_t e = w & 0x33333333u;         // nibbles: codes of dims 0,2,4,..,14
  const uint32_t o = (w >> 2) & 0x33333333u;  // nibbles: codes of dims 1,3,5,..,15
  const uint32_t sel[4] = {e, e >> 16, o, o >> 16};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = prmt(x, 0u, sel[i]);  // low bytes of the 4 selected values
    const uint32_t hi = prmt(y, 0u, sel[i]);  // high bytes
    r[2 * i] = prmt(lo, hi, 0x5140u);
    r[2 * i + 1] = prmt(lo, hi, 0x7362u);
  }
}

// tc_lut_word's registers in the K column order: dims (0,2) (1,3) (4,6) (5,7) ..
OSCAR_DEVINL void tc_k_order(const uint32_t* in, uint32_t* out) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    out[2 * m] = in[m];
    out[2 * m + 1] = in[4 + m];
  }
}

// 16 fp32 values of dims 16j..16j+15 -> 8 registers in the same permuted order,
// through the chain T(fp16(x)) (K) or its fp16 bit pattern (V)
template <typename T, bool kV>
OSCAR_DEVINL void tc_pack_word(const float* src, bool live, uint32_t* r) {
  float f[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 q = live ? *reinterpret_cast<const float4*>(src + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
    f[4 * i] = q.x;
    f[4 * i + 1] = q.y;
    f[4 * i + 2] = q.z;
    f[4 * i + 3] = q.w;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d0 = (i < 4) ? 4 * i : 4 * (i - 4) + 1;  // dims (d0, d0 + 2)
    if (kV)
      r[i] = pack2<__half>(chain_f16<T>(f[d0]), chain_f16<T>(f[d0 + 2]));
    else
      r[i] = pack2<T>(chain<T>(f[d0]), chain<T>(f[d0 + 2]));
  }
}

// 4-entry value tables from a token's fp16 (scale, zero) pair, built with
// packed conversions: K holds T(fp16(c * s + z)) (c * s + z computed as one fma:
// c * s is exact), V the fp16 bit patterns of the same values clamped to the
// fp16 range (make_klut / make_vlut semantics)
template <typename T>
OSCAR_DEVINL uint2 tc_klut(uint32_t meta) {
  const float sc = f16_bits_to_f32(meta & 0xffffu), zr = f16_bits_to_f32(meta >> 16);
  __half2 h01 = __floats2half2_rn(zr, fmaf(1.0f, sc, zr)), h23 = __floats2half2_rn(fmaf(2.0f, sc, zr), fmaf(3.0f, sc, zr));
  uint32_t p01, p23;
  if (std::is_same<T, __nv_bfloat16>::value) {
    const float2 g01 = __half22float2(h01), g23 = __half22float2(h23);
    const __nv_bfloat162 b01 = __floats2bfloat162_rn(g01.x, g01.y), b23 = __floats2bfloat162_rn(g23.x, g23.y);
    p01 = *reinterpret_cast<const uint32_t*>(&b01);
    p23 = *reinterpret_cast<const uint32_t*>(&b23);
  } else {
    p01 = *reinterpret_cast<const uint32_t*>(&h01);
    p23 = *reinterpret_cast<const uint32_t*>(&h23);
  }
  return lut_from(p01, p23);
}
template <typename T>
OSCAR_DEVINL uint2 tc_vlut(uint32_t meta) {
  const float sc = f16_bits_to_f32(meta & 0xffffu), zr = f16_bits_to_f32(meta >> 16);
  const __half2 h01 = __floats2half2_rn(zr, fmaf(1.0f, sc, zr)), h23 = __floats2half2_rn(fmaf(2.0f, sc, zr), fmaf(3.0f, sc, zr));
  float2 g01 = __half22float2(h01), g23 = __half22float2(h23);
  if (std::is_same<T, __nv_bfloat16>::value) {
    g01 = __bfloat1622float2(__floats2bfloat162_rn(g01.x, g01.y));
    g23 = __bfloat1622float2(__floats2bfloat162_rn(g23.x, g23.y));
  }
  const __half2 c01 = __floats2half2_rn(fminf(fmaxf(g01.x, -65504.0f), 65504.0f), fminf(fmaxf(g01.y, -65504.0f), 65504.0f));
  const __half2 c23 = __floats2half2_rn(fminf(fmaxf(g23.x, -65504.0f), 65504.0f), fminf(fmaxf(g23.y, -65504.0f), 65504.0f));
  return lut_from(*reinterpret_cast<const uint32_t*>(&c01), *reinterpret_cast<const uint32_t*>(&c23));
}

OSCAR_DEVINL float tc_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// order-preserving float <-> int map (for redux.sync max)
OSCAR_DEVINL int tc_ord(float v) {
  const int k = __float_as_int(v);
  return k >= 0 ? k : k ^ 0x7fffffff;
}
OSCAR_DEVINL float tc_unord(int k) { return __int_as_float(k >= 0 ? k : k ^ 0x7fffffff); }

// TMA of INT2 stage s into ring slot s & 1: four 48-byte boxes (K [0,48),
// K [48,96), V [0,48), V [16,64)) of `rows` tokens per page of the stage, and
// (with a staging window) the owner tags of the same seats by one bulk copy.
// `parts`: kTcBoxes (the boxes, and the transaction count of the whole stage),
// kTcTags (the owner tags), or both.
constexpr int kTcBoxes = 1, kTcTags = 2;
OSCAR_DEVINL void tc_issue_stage(TcSmem& sm, const AttnArgs& a, int s, int lo, int hi, int bs_log2, int page0, int h,
                                 const CUtensorMap* tmk, const CUtensorMap* tmv, uint32_t b_full,
                                 int parts = kTcBoxes | kTcTags) {
  const int bs = 1 << bs_log2;
  const int rows_box = min(bs, kTcStage);
  const int slot = s & 1;
  const int base = lo + s * kTcStage;
  const int end = min(base + kTcStage, hi);
  const int pg_first = base >> bs_log2, pg_last = (end - 1) >> bs_log2;
  const uint32_t bar = b_full + 8 * slot;
  const bool tags = a.owner != nullptr;
  if (parts & kTcBoxes)
    tc::mbar_expect_tx(bar, (uint32_t)((pg_last - pg_first + 1) * rows_box * (4 * kTcRow + (tags ? 8 : 0))));
  for (int pg = pg_first; pg <= pg_last; ++pg) {
    const int blk = sm.btab[pg - page0];
    const int off0 = (bs > kTcStage) ? base - (pg << bs_log2) : 0;
    const int row = (pg << bs_log2) + off0 - base;
    const int y = (blk << bs_log2) + off0;
    const int xk = (int)(h * a.ksh), xv = (int)(h * a.vsh);
    if (parts & kTcBoxes) {
      tc::tma_load_2d(smem_u32(&sm.ka[slot][row][0]), tmk, xk, y, bar);
      tc::tma_load_2d(smem_u32(&sm.kb[slot][row][0]), tmk, xk + 48, y, bar);
      tc::tma_load_2d(smem_u32(&sm.va[slot][row][0]), tmv, xv, y, bar);
      tc::tma_load_2d(smem_u32(&sm.vb[slot][row][0]), tmv, xv + 16, y, bar);
    }
    if (tags && (parts & kTcTags))
      tc::bulk_load(smem_u32(&sm.own[slot][row]), a.owner + (int64_t)(blk % (int)a.stage_rows) * bs + off0,
                    (uint32_t)rows_box * 8u, bar);
  }
}

struct TcWait {
  int* abort;
  // bounded wait; after a timeout (or once the CTA gave up) every wait returns
  // at once, so control flow stays uniform and the kernel drains and exits
  OSCAR_DEVINL void operator()(uint32_t bar, uint32_t parity) const {
    if (tc::mbar_try(bar, parity)) return;
    if (*reinterpret_cast<volatile int*>(abort)) return;
    if (!tc::mbar_wait(bar, parity)) {
      *reinterpret_cast<volatile int*>(abort) = 1;
      flag_error(16u);
    }
  }
};

// staged index j of this CTA's groups -> fp32 row offset of its seat (and its
// position): the last group whose prefix count is <= j holds it
OSCAR_DEVINL int64_t tc_staged_row(const TcSmem& sm, const AttnArgs& a, int j, int ngroups, int sp, int nsplit,
                                   int req, int bs_log2, int h, int* pos_out) {
  int lo_w = 0, hi_w = ngroups - 1;
  while (lo_w < hi_w) {
    const int mid = (lo_w + hi_w + 1) >> 1;
    if (sm.gpref[mid] <= j) lo_w = mid; else hi_w = mid - 1;
  }
  const int bit = (int)__fns(sm.gmask[lo_w], 0u, j - sm.gpref[lo_w] + 1);
  const int pos = (sp + lo_w * nsplit) * 32 + bit;
  const int blk = a.bt[(int64_t)req * a.bt_stride + (pos >> bs_log2)];
  const int64_t seat = (int64_t)(blk % (int)a.stage_rows) * a.bs + (pos & (a.bs - 1));
  *pos_out = pos;
  return (seat * a.hk + h) * 256;
}

// staged K rows of a warp's 32 tokens (one per lane: row_off, live) into its
// TMEM lane quarter at t_a (64 columns: 128 dims as fp16/bf16 pairs).
// tcgen05.st.16x256b: thread i writes lanes i / 4 and 8 + i / 4 of a 16-lane
// half, columns 2 (i % 4), + 1 of each 16-dim group: (dims 4m, 4m+2), (4m+1,
// 4m+3).  src points at dims 4 (lane % 4) of the thread's 128-dim half; a load
// instruction covers 8 tokens x 64 contiguous bytes; dead tokens get zeros.
template <typename T>
OSCAR_DEVINL void tc_staged_k(uint32_t t_a, const float* src, int64_t row_off, bool live, int lane) {
#pragma unroll 1
  for (int hb = 0; hb < 2; ++hb) {
    const int la = 16 * hb + (lane >> 2), lb = la + 8;
    const int64_t ra = __shfl_sync(0xffffffffu, row_off, la), rb = __shfl_sync(0xffffffffu, row_off, lb);
    const bool va = __shfl_sync(0xffffffffu, (int)live, la) != 0;
    const bool vb = __shfl_sync(0xffffffffu, (int)live, lb) != 0;
    if (!__any_sync(0xffffffffu, vb)) {
      // lanes 8..15 of the half are dead: one pass of 8 loads
      float4 xs[8];
#pragma unroll
      for (int g = 0; g < 8; ++g)
        xs[g] = va ? __ldg(reinterpret_cast<const float4*>(src + ra + 16 * g)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        uint32_t r[16];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const float4 x = xs[4 * cb + g];
          r[4 * g] = pack2<T>(chain<T>(x.x), chain<T>(x.z));
          r[4 * g + 1] = pack2<T>(chain<T>(x.y), chain<T>(x.w));
          r[4 * g + 2] = 0u;
          r[4 * g + 3] = 0u;
        }
        tc::tmem_st16x256_x4(t_a + ((uint32_t)(16 * hb) << 16) + 32 * cb, r);
      }
    } else {
#pragma unroll 1
      for (int cb = 0; cb < 2; ++cb) {
        float4 xs[4], ys[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int off = 16 * (4 * cb + g);
          xs[g] = va ? __ldg(reinterpret_cast<const float4*>(src + ra + off)) : make_float4(0.f, 0.f, 0.f, 0.f);
          ys[g] = vb ? __ldg(reinterpret_cast<const float4*>(src + rb + off)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        uint32_t r[16];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          r[4 * g] = pack2<T>(chain<T>(xs[g].x), chain<T>(xs[g].z));
          r[4 * g + 1] = pack2<T>(chain<T>(xs[g].y), chain<T>(xs[g].w));
          r[4 * g + 2] = pack2<T>(chain<T>(ys[g].x), chain<T>(ys[g].z));
          r[4 * g + 3] = pack2<T>(chain<T>(ys[g].y), chain<T>(ys[g].w));
        }
        tc::tmem_st16x256_x4(t_a + ((uint32_t)(16 * hb) << 16) + 32 * cb, r);
      }
    }
  }
}

// staged V rows of a warp's 32 tokens into V^T (fp16).  vt_q points at the
// warp's first token group, + 4 lane; the V^T word of (token, dims 4m, 4m+2)
// sits at row group 2g, (4m+1, 4m+3) at 2g+1, so the 8 tokens x 4 words of an
// instruction are 128 contiguous bytes.
template <typename T>
OSCAR_DEVINL void tc_staged_v(uint8_t* vt_q, const float* src, int64_t row_off, bool live, int lane) {
#pragma unroll 1
  for (int o = 0; o < 4; ++o) {
    const int lt = 8 * o + (lane >> 2);
    const int64_t rt = __shfl_sync(0xffffffffu, row_off, lt);
    const bool vt = __shfl_sync(0xffffffffu, (int)live, lt) != 0;
    float4 xs[8];
#pragma unroll
    for (int g = 0; g < 8; ++g)
      xs[g] = vt ? __ldg(reinterpret_cast<const float4*>(src + rt + 16 * g)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t* dst = reinterpret_cast<uint32_t*>(vt_q + o * 128 + (2 * g) * kTcVtSbo);
      dst[0] = pack2<__half>(chain_f16<T>(xs[g].x), chain_f16<T>(xs[g].z));
      dst[kTcVtSbo / 4] = pack2<__half>(chain_f16<T>(xs[g].y), chain_f16<T>(xs[g].w));
    }
  }
}

template <typename T>
__global__ void __maxnreg__(72)
    decode_tc_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv) {
  constexpr int D = 256;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // grid (kv heads, items): the hardware starts CTAs x-fastest, so every head of the
  // heaviest requests (planned first) starts before the light ones
  const int item = blockIdx.y, h = blockIdx.x;
  const int ri = find_bucket(p.item_begin, p.num_req, item);
  const int sp = item - p.item_begin[ri];
  const int req = p.req_id[ri];
  const int q_start = p.q_start[ri], qlen = p.q_len[ri], seq = p.seq[ri], prefix = p.prefix[ri];
  const int G = a.group;
  const int R = qlen * G;
  const int lo = sp * p.chunk[ri];
  const int hi = min(lo + p.chunk[ri], prefix);
  const int bs = a.bs;
  const int bs_log2 = 31 - __clz(bs);
  const int n_int = (hi > lo) ? (hi - lo + kTcStage - 1) / kTcStage : 0;  // INT2 stages
  const int page0 = lo >> bs_log2;
  const int npages = (hi > lo) ? ((hi - 1) >> bs_log2) - page0 + 1 : 0;
  const int nsplit = p.splits[ri];
  const int ngroups32 = (prefix + 31) >> 5;
  const int ngroups = min(sp < ngroups32 ? (ngroups32 - 1 - sp) / nsplit + 1 : 0, kTcMaxWords);
  constexpr int kWarps = kTcCompute / 32;

  const uint32_t b_full = smem_u32(&sm.bar_full[0]), b_empty = smem_u32(&sm.bar_empty[0]);
  const uint32_t b_k = smem_u32(&sm.bar_k[0]), b_s = smem_u32(&sm.bar_s[0]), b_v = smem_u32(&sm.bar_v[0]),
                 b_p = smem_u32(&sm.bar_p[0]), b_pv = smem_u32(&sm.bar_pv[0]);
  const TcWait wait{&sm.abort};

  // ---------------- prologue.  Programmatic dependent launch: this grid may
  // start while the kernels in front of it (the write step, the rotation)
  // still run.  Before waiting for them, the producer warp sets up barriers,
  // TMEM and the page slice and issues the TMA boxes of the first two INT2
  // stages: the block table is the engine's input and the history below the
  // prefix was written by earlier steps, so none of it depends on those
  // kernels.  After the wait: the owner tags (the write step updates them), Q
  // (the rotation writes it) and the staged-group scan.  Staged stages run
  // first, so their fp32 loads overlap the TMA of the first INT2 stages.
  if (warp == kTcProdWarp) {
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        tc::mbar_init(b_full + 8 * i, 1);
        tc::mbar_init(b_empty + 8 * i, kWarps);           // every dequant warp read the slot
        tc::mbar_init(b_k + 8 * i, kWarps / 2 + kTcSmWarps);  // K warps wrote A_K, softmax warps freed S
        tc::mbar_init(b_s + 8 * i, 1);
        tc::mbar_init(b_v + 8 * i, kWarps / 2);            // V warps wrote V^T
        tc::mbar_init(b_p + 8 * i, kTcSmWarps);            // softmax warps wrote P^T
        tc::mbar_init(b_pv + 8 * i, 1);
      }
      sm.abort = 0;
      tc::mbar_fence_init();
    }
    for (int i = lane; i < npages; i += 32) {
      int blk = a.bt[(int64_t)req * a.bt_stride + page0 + i];
      if (blk < 0 || blk >= a.num_blocks) {
        flag_error(2u);
        blk = 0;
      }
      sm.btab[i] = blk;
    }
    tc::tmem_alloc(smem_u32(&sm.tmem), kTcCols);
    tc::tmem_relinquish();
    __syncwarp();
    if (tc::elect_one()) {
      for (int s = 0; s < min(2, n_int); ++s)
        tc_issue_stage(sm, a, s, lo, hi, bs_log2, page0, h, &tmk, &tmv, b_full, kTcBoxes);
    }
    __syncwarp();
  } else if (warp >= kTcDeqWarps) {
    // softmax warps: row maxima start at -inf; P^T starts zeroed, so the rows
    // >= R that the softmax never writes hold zeros
    const int st_tid = tid - kTcCompute;
    if (st_tid < kTcQuarters * kTcRows) (&sm.mrow[0][0])[st_tid] = -INFINITY;
    for (int i = st_tid; i < (int)(sizeof(sm.pt) / 16); i += 32 * kTcSmWarps)
      reinterpret_cast<uint4*>(&sm.pt[0][0])[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  // dequant warps: the block-table entries of this CTA's staged-group scan (first
  // batch: groups k = warp + 16 u), an engine input read before the wait
  constexpr int kScanPer = 4;
  int gblk[kScanPer];
  bool ghit[kScanPer];
#pragma unroll
  for (int u = 0; u < kScanPer; ++u) {
    gblk[u] = -1;
    ghit[u] = false;
    const int k = warp + u * kWarps, pos = (sp + k * nsplit) * 32 + lane;
    if (warp < kTcDeqWarps && a.owner != nullptr && k < ngroups && pos < prefix) {
      gblk[u] = a.bt[(int64_t)req * a.bt_stride + (pos >> bs_log2)];
      if (gblk[u] >= a.num_blocks) gblk[u] = -1;
    }
  }
  pdl_wait();
  if (warp == kTcProdWarp) {
    if (a.owner != nullptr && tc::elect_one()) {
      for (int s = 0; s < min(2, n_int); ++s)
        tc_issue_stage(sm, a, s, lo, hi, bs_log2, page0, h, &tmk, &tmv, b_full, kTcTags);
    }
    __syncwarp();
  } else if (warp < kTcDeqWarps) {
    if (tid < kTcRows) sm.lim[tid] = tid < R ? seq - qlen + tid / G + 1 : INT_MIN;
    // Q rows n < R, 16-dim word j: k-group 2j holds dims 16j + {0,2,1,3,4,6,5,7}, 2j+1 dims
    // 16j + {8,10,9,11,12,14,13,15} (the K column order); k-groups 32, 33 hold the bias
    // column: 1 at k = 256, zeros after.  Items u = tid, tid + 512: their loads and the
    // owner tags of the scan's first batch go out in one round.
    constexpr int kQItems = (kTcRows * 17 + kTcCompute - 1) / kTcCompute;
    uint4 qraw[kQItems][2];
#pragma unroll
    for (int i = 0; i < kQItems; ++i) {
      const int u = tid + i * kTcCompute, n = u / 17, j = u - 17 * (u / 17);
      qraw[i][0] = qraw[i][1] = make_uint4(0, 0, 0, 0);
      if (u < kTcRows * 17 && j < 16 && n < R) {
        const T* qrow =
            reinterpret_cast<const T*>(a.q) + ((int64_t)(q_start + n / G) * a.hq + (int64_t)h * G + n % G) * D;
        qraw[i][0] = *reinterpret_cast<const uint4*>(qrow + 16 * j);
        qraw[i][1] = *reinterpret_cast<const uint4*>(qrow + 16 * j + 8);
      }
    }
    // this CTA's groups of the whole request, g = sp + k * nsplit: up to four per
    // warp (block-table entries first, then the owner tags), kept in registers until
    // the prefix counts give each staged position its index j; the first staged
    // stage's rows and positions (j < 128) then go to srow / spos
    const bool scan_all = ngroups <= kScanPer * kWarps;
    auto scan_tags = [&](int k0) {
      int64_t tag[kScanPer];
#pragma unroll
      for (int u = 0; u < kScanPer; ++u) {
        const int k = k0 + u * kWarps, pos = (sp + k * nsplit) * 32 + lane;
        tag[u] = gblk[u] >= 0 ? a.owner[(int64_t)(gblk[u] % (int)a.stage_rows) * bs + (pos & (bs - 1))] : -2;
      }
#pragma unroll
      for (int u = 0; u < kScanPer; ++u) {
        const int k = k0 + u * kWarps;
        ghit[u] = gblk[u] >= 0 && tag[u] == (int64_t)gblk[u];
        const uint32_t bits = __ballot_sync(0xffffffffu, ghit[u]);
        if (lane == 0 && k < ngroups) sm.gmask[k] = bits;
      }
    };
    if (warp < ngroups) scan_tags(warp);
#pragma unroll
    for (int i = 0; i < kQItems; ++i) {
      const int u = tid + i * kTcCompute, n = u / 17, j = u - 17 * (u / 17);
      if (u >= kTcRows * 17) break;
      uint4 ev = make_uint4(0, 0, 0, 0), od = ev;
      if (j == 16) {
        ev.x = (uint32_t)(std::is_same<T, __nv_bfloat16>::value ? 0x3F80u : 0x3C00u);  // 1.0 in T
      } else {
        const uint4 q0 = qraw[i][0], q1 = qraw[i][1];
        ev = make_uint4(prmt(q0.x, q0.y, 0x5410u), prmt(q0.x, q0.y, 0x7632u), prmt(q0.z, q0.w, 0x5410u),
                        prmt(q0.z, q0.w, 0x7632u));
        od = make_uint4(prmt(q1.x, q1.y, 0x5410u), prmt(q1.x, q1.y, 0x7632u), prmt(q1.z, q1.w, 0x5410u),
                        prmt(q1.z, q1.w, 0x7632u));
      }
      uint8_t* dst = sm.qb + (n >> 3) * kTcQSbo + (2 * j) * 128 + (n & 7) * 16;
      *reinterpret_cast<uint4*>(dst) = ev;
      *reinterpret_cast<uint4*>(dst + 128) = od;
    }
    // later batches (histories with more groups than one pass holds)
    for (int k0 = warp + kScanPer * kWarps; k0 < ngroups; k0 += kScanPer * kWarps) {
#pragma unroll
      for (int u = 0; u < kScanPer; ++u) {
        const int k = k0 + u * kWarps, pos = (sp + k * nsplit) * 32 + lane;
        gblk[u] = -1;
        if (a.owner != nullptr && k < ngroups && pos < prefix) {
          gblk[u] = a.bt[(int64_t)req * a.bt_stride + (pos >> bs_log2)];
          if (gblk[u] >= a.num_blocks) gblk[u] = -1;
        }
      }
      scan_tags(k0);
    }
    if (tid < kTcStage) {
      sm.srow[tid] = -1;
      sm.spos[tid] = hi;
    }
    tc::bar_sync(5, kTcCompute);  // gmask ready
    if (warp == 0) {
      int run = 0;
      for (int w0 = 0; w0 < ngroups; w0 += 32) {
        const int wi = w0 + lane;
        const int c = (wi < ngroups) ? __popc(sm.gmask[wi]) : 0;
        int incl = c;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, d);
          if (lane >= d) incl += y;
        }
        if (wi < ngroups) sm.gpref[wi] = run + incl - c;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) {
        sm.gpref[ngroups] = run;
        sm.n_staged = run;
      }
    }
    tc::bar_sync(5, kTcCompute);  // gpref ready
    if (scan_all) {
      // the registers hold this warp's (only) batch of groups
#pragma unroll
      for (int u = 0; u < kScanPer; ++u) {
        const int k = warp + u * kWarps;
        if (k < ngroups && ghit[u]) {
          const int j = sm.gpref[k] + __popc(sm.gmask[k] & ((1u << lane) - 1u));
          if (j < kTcStage) {
            const int pos = (sp + k * nsplit) * 32 + lane;
            const int64_t seat = (int64_t)(gblk[u] % (int)a.stage_rows) * bs + (pos & (bs - 1));
            const int slot = (j & 3) * 32 + (j >> 2);  // token slot of staged index j
            sm.srow[slot] = (seat * a.hk + h) * D;
            sm.spos[slot] = pos;
          }
        }
      }
    } else if (tid < kTcStage) {
      // more groups than one pass holds: search the prefix counts
      const int j = (tid & 31) * 4 + (tid >> 5);
      if (j < sm.n_staged) {
        int lo_w = 0, hi_w = ngroups - 1;  // last group whose prefix count is <= j
        while (lo_w < hi_w) {
          const int mid = (lo_w + hi_w + 1) >> 1;
          if (sm.gpref[mid] <= j) lo_w = mid; else hi_w = mid - 1;
        }
        const int bit = (int)__fns(sm.gmask[lo_w], 0u, j - sm.gpref[lo_w] + 1);
        const int pos = (sp + lo_w * nsplit) * 32 + bit;
        const int blk = a.bt[(int64_t)req * a.bt_stride + (pos >> bs_log2)];
        const int64_t seat = (int64_t)(blk % (int)a.stage_rows) * bs + (pos & (bs - 1));
        sm.srow[tid] = (seat * a.hk + h) * D;
        sm.spos[tid] = pos;
      }
    }
  }
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  // the split merge may be scheduled now: it waits for this grid before reading partials
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const uint32_t tmem = sm.tmem;
  const int n_staged = sm.n_staged;
  const int n_sst = (n_staged + kTcStage - 1) / kTcStage;  // staged stages, run first
  const int nst = n_sst + n_int;

  if (warp == kTcProdWarp) {
    // ============================ producer + MMA issuer
    // an event loop over three independent queues, none of which blocks the
    // others: QK(qs) once A_K[qs & 1] is written and S[qs & 1] is free; PV(ps)
    // once V^T and P^T of stage ps are written; the TMA of INT2 stage rf once
    // its ring slot is empty.  (Each barrier's next phase needs this warp's
    // own next issue, so a test of the current parity is never ambiguous.)
    // The whole warp runs the loop (lane 0's test results are broadcast, so
    // control flow stays warp-uniform); one elected lane issues.
    constexpr uint32_t idesc_qk = tc::instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u, 0, 0, 128, kTcRows);
    constexpr uint32_t idesc_pv = tc::instr_desc(0u, 1, 1, 128, kTcRows);
    constexpr uint32_t idesc_l = tc::instr_desc(0u, 0, 1, 128, kTcRows);  // ones (TMEM) x P^T: row sums
    // descriptors of k-step 0; k-step j starts 256 * j bytes later (+16 * j in the start field);
    // buffer 1 of V^T / P^T sits sizeof(vt[0]) / sizeof(pt[0]) bytes after buffer 0
    const uint64_t dq0 = tc::smem_desc(smem_u32(sm.qb), 128, kTcQSbo);
    const uint64_t dv0 = tc::smem_desc(smem_u32(sm.vt[0]), 128, kTcVtSbo);
    const uint64_t dp0 = tc::smem_desc(smem_u32(sm.pt[0]), 128, kTcVtSbo);
    uint32_t idle = 0;
    for (int qs = 0, ps = 0, rf = 2; ps < nst;) {
      bool prog = false;
      if (ps < qs && __shfl_sync(0xffffffffu, (int)(tc::mbar_test(b_v + 8 * (ps & 1), (ps >> 1) & 1) &&
                                                  tc::mbar_test(b_p + 8 * (ps & 1), (ps >> 1) & 1)), 0)) {
        // PV of stage ps from V^T[ps & 1], P^T[ps & 1]
        tc::tc_fence_after();
        const uint64_t dva = dv0 + (uint64_t)((ps & 1) * (sizeof(sm.vt[0]) >> 4));
        const uint64_t dvb = dva + (16 * kTcVtSbo >> 4);
        const uint64_t dpa = dp0 + (uint64_t)((ps & 1) * (sizeof(sm.pt[0]) >> 4));
        const uint32_t d_o = tmem + kTcColO;
        const uint32_t acc0 = ps > 0 ? 1u : 0u;
        if (tc::elect_one()) {
#pragma unroll
          for (int j = 0; j < kTcStage / 16; ++j) {
            tc::mma_ss(d_o, dva + 16 * j, dpa + 16 * j, idesc_pv, j > 0 ? 1u : acc0);
            tc::mma_ss(d_o + 32, dvb + 16 * j, dpa + 16 * j, idesc_pv, j > 0 ? 1u : acc0);
            // the row sums of P accumulate beside O, from the same fp16 P (every lane of L
            // holds them; one 16-token block of ones serves every k-step).  The tensor
            // pipe has room for them: its cost per MMA is the same at N = 32 as at 64,
            // and the softmax warps, not the MMAs, bound a stage.
            tc::mma_ts(tmem + kTcColL, tmem + kTcColOnes, dpa + 16 * j, idesc_l, j > 0 ? 1u : acc0);
          }
          tc::mma_commit(b_pv + 8 * (ps & 1));
        }
        __syncwarp();
        ++ps;
        prog = true;
      }
      if (qs < nst && __shfl_sync(0xffffffffu, (int)tc::mbar_test(b_k + 8 * (qs & 1), (qs >> 1) & 1), 0)) {
        // QK of stage qs into S[qs & 1] from A_K[qs & 1]
        tc::tc_fence_after();
        const uint32_t d_s = tmem + kTcColS + 32 * (qs & 1), a_k = tmem + ((qs & 1) ? kTcColA1 : kTcColA0);
        if (tc::elect_one()) {
#pragma unroll
          for (int j = 0; j < kTcK / 16; ++j) tc::mma_ts(d_s, a_k + 8 * j, dq0 + 16 * j, idesc_qk, j > 0 ? 1u : 0u);
          tc::mma_commit(b_s + 8 * (qs & 1));
        }
        __syncwarp();
        ++qs;
        prog = true;
      }
      if (rf < n_int && __shfl_sync(0xffffffffu, (int)tc::mbar_test(b_empty + 8 * (rf & 1), ((rf - 2) >> 1) & 1), 0)) {
        // ring slot rf & 1 was read by every dequant warp (INT2 stage rf - 2)
        if (tc::elect_one()) tc_issue_stage(sm, a, rf, lo, hi, bs_log2, page0, h, &tmk, &tmv, b_full);
        __syncwarp();
        ++rf;
        prog = true;
      }
      if (prog) {
        idle = 0;
      } else if (__shfl_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&sm.abort), 0) != 0) {
        break;  // another warp timed out: drain
      } else if (++idle > 4 * tc::kSpinLimit) {
        if (lane == 0) {
          *reinterpret_cast<volatile int*>(&sm.abort) = 1;
          flag_error(16u);
        }
        break;
      }
    }
  } else if (warp < kTcDeqWarps) {
    // ============================ dequant warps.  Warp w serves the 32 tokens of
    // TMEM lane quarter w % 4 (tok = 32 (w % 4) + lane) in role q = w / 4: K dims
    // [0, 128) (q = 0), K dims [128, 256) (1), V dims [0, 128) (2), V dims
    // [128, 256) (3).  K goes into TMEM (A operand), V into V^T in shared memory;
    // the softmax runs in its own warps, so these warps only dequantise.
    const int q = warp >> 2, tok = tid & 127;
    const bool is_k = q < 2;
    const int half = q & 1;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t neg_inf = std::is_same<T, __nv_bfloat16>::value ? 0xFF80u : 0xFC00u;
    // this thread's 32 code bytes as two 16-byte pieces of the raw rows (offsets
    // from ka[slot][tok]; kb / va / vb follow ka at fixed distances):
    //   K half 0: K bytes [32, 64) = ka[32, 48) + kb[0, 16);  K half 1: K bytes [64, 96) = kb[16, 48)
    //   V half 0: V bytes [0, 32)  = va[0, 32);              V half 1: V bytes [32, 64) = vb[16, 48)
    constexpr int kKb = (int)(offsetof(TcSmem, kb) - offsetof(TcSmem, ka));
    constexpr int kVa = (int)(offsetof(TcSmem, va) - offsetof(TcSmem, ka));
    constexpr int kVb = (int)(offsetof(TcSmem, vb) - offsetof(TcSmem, ka));
    const int off0 = (q == 0) ? 32 : (q == 1) ? kKb + 16 : (q == 2) ? kVa : kVb + 16;
    const int off1 = (q == 0) ? kKb : (q == 1) ? kKb + 32 : (q == 2) ? kVa + 16 : kVb + 32;
    const int meta_off = is_k ? 0 : 4;  // K (scale, zero) at slot bytes [0, 4), V at [4, 8)
    const int vt_off = (16 * half) * kTcVtSbo + (tok >> 3) * 128 + (tok & 7) * 16;

    for (int it = 0; it < nst; ++it) {
      const int b = it & 1;
      const uint32_t t_a = tmem + lane_base + (b ? kTcColA1 : kTcColA0) + 64 * half;
      // A_K[b] was last read by the QK of stage it - 2, V^T[b] by its PV
      auto wait_out = [&]() {
        if (it >= 2) {
          if (is_k) wait(b_s + 8 * b, ((it - 2) >> 1) & 1);
          else wait(b_pv + 8 * b, ((it - 2) >> 1) & 1);
          tc::tc_fence_after();
        }
      };
      bool live;
      if (it >= n_sst) {
        const int ii = it - n_sst;  // INT2 stage
        const int slot = ii & 1;
        const int pos = lo + ii * kTcStage + tok;
        wait(b_full + 8 * slot, (ii >> 1) & 1);
        const uint8_t* raw = &sm.ka[slot][tok][0];
        const uint32_t meta = *reinterpret_cast<const uint32_t*>(raw + meta_off);
        const uint4 c0 = *reinterpret_cast<const uint4*>(raw + off0);
        const uint4 c1 = *reinterpret_cast<const uint4*>(raw + off1);
        live = pos < hi;
        if (live && a.owner != nullptr) live = sm.own[slot][tok] != (int64_t)sm.btab[(pos >> bs_log2) - page0];
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(b_empty + 8 * slot);
        uint2 lut = make_uint2(0, 0);
        if (live) lut = is_k ? tc_klut<T>(meta) : tc_vlut<T>(meta);
        const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        // (the ring slot is released before waiting for the output buffer, so the
        // next TMA into it does not wait for the slowest consumer's PV / QK)
        wait_out();
        if (is_k) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            uint32_t r[32];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t v[8];
              tc_lut_word(cw[4 * g + j], lut.x, lut.y, v);
              tc_k_order(v, r + 8 * j);
            }
            tc::tmem_st32(t_a + 32 * g, r);
          }
        } else {
          uint8_t* vt_row = sm.vt[b] + vt_off;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint32_t r[8];
            tc_lut_word(cw[j], lut.x, lut.y, r);
            *reinterpret_cast<uint4*>(vt_row + (2 * j) * kTcVtSbo) = make_uint4(r[0], r[1], r[2], r[3]);
            *reinterpret_cast<uint4*>(vt_row + (2 * j + 1) * kTcVtSbo) = make_uint4(r[4], r[5], r[6], r[7]);
          }
        }
      } else {
        // staged stage: the j-th staged position of this CTA's groups (fp32 rows);
        // consecutive j go to different lane quarters, so a partial stage
        // spreads its loads over all sixteen warps
        const int j = it * kTcStage + (tok & 31) * 4 + (tok >> 5);
        live = j < n_staged;
        wait_out();
        int64_t row_off = 0;
        if (it == 0) {
          row_off = live ? sm.srow[tok] : 0;  // located in the prologue
        } else if (live) {
          int pos;
          row_off = tc_staged_row(sm, a, j, ngroups, sp, nsplit, req, bs_log2, h, &pos);
        }
        // coalesced fp32 loads: a thread reads 16 bytes (dims 4 (lane % 4) .. + 3 of a 16-dim
        // group) of the token of lane lane / 4 (+ 8, 16, 24) of the quarter, so each
        // instruction covers 8 tokens x 64 contiguous bytes; dead tokens get zeros
        const float* src = (is_k ? a.stage_k : a.stage_v) + 128 * half + 4 * (lane & 3);
        if (is_k) {
          tc_staged_k<T>(t_a, src, row_off, live, lane);
        } else {
          tc_staged_v<T>(sm.vt[b] + (16 * half) * kTcVtSbo + ((warp & 3) * 4) * 128 + 4 * lane, src, row_off, live,
                         lane);
        }
      }
      if (is_k) {
        if (q == 0) {
          // bias k-step (columns 128..135): element 256 = 0 for live tokens, -inf for masked ones
          const uint32_t bias[8] = {live ? 0u : neg_inf, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
          tc::tmem_st8(t_a + 128, bias);
        }
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(b_k + 8 * b);
      } else {
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(b_v + 8 * b);
      }
    }
  } else {
    // ============================ softmax warps.  Warp 16 + 4 hr + lq serves the
    // tokens of TMEM lane quarter lq, one token per thread, for query rows
    // 16 hr .. 16 hr + 15: it reads the token's scores from S^T (lane = token,
    // column = row), keeps the running row maxima (a copy per warp, in
    // sm.mrow) and writes the token's P^T column; the row sums of P come from
    // the tensor cores (L beside O), so O and l see the same fp16 P.  A half
    // with no query row (16 hr >= R) keeps only the barrier protocol.  The
    // running maximum moves only when a score exceeds it by more than 15 (log2
    // units): P stays <= 2^15 in fp16, and O / l are rescaled on those stages
    // only.  The four warps of a half vote and reduce on named barrier 1 + hr.
    const int lq = (warp - kTcDeqWarps) & 3, hr = (warp - kTcDeqWarps) >> 2, tok = 32 * lq + lane;
    const uint32_t lane_base = (uint32_t)(32 * lq) << 16;
    const bool need_lim = hi > seq - qlen + 1;  // history reaches the causal window (cache-only chunks)
    const float scale = a.scale_log2;
    const bool active = 16 * hr < R;
    const int pt_off = (tok >> 3) * 128 + (tok & 7) * 16;
    if (hr == 0) {
      // the ones block of the row-sum MMA (fp16 1.0 pairs), this quarter's lanes
      const uint32_t ones[8] = {0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u,
                                0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u};
      tc::tmem_st8(tmem + lane_base + kTcColOnes, ones);
      tc::tmem_wait_st();
      tc::tc_fence_before();
    }
    // S[0] and S[1] are free for the QKs of stages 0 and 1
    if (lane == 0) {
      tc::mbar_arrive(b_k);
      tc::mbar_arrive(b_k + 8);
    }
    for (int st = 0; st < nst; ++st) {
      const int b = st & 1;
      int pos = hi;  // position of this thread's token (for the causal limit of cache-only chunks)
      if (need_lim && active) {
        if (st >= n_sst) {
          pos = lo + (st - n_sst) * kTcStage + tok;
        } else {
          const int j = st * kTcStage + (tok & 31) * 4 + (tok >> 5);
          if (st == 0) pos = sm.spos[tok];
          else if (j < n_staged) tc_staged_row(sm, a, j, ngroups, sp, nsplit, req, bs_log2, h, &pos);
        }
      }
      wait(b_s + 8 * b, (st >> 1) & 1);
      tc::tc_fence_after();
      if (st >= 2) {
        // P^T[b] was last read by the PV of stage st - 2
        wait(b_pv + 8 * b, ((st - 2) >> 1) & 1);
      }
      if (active) {
        // the token's scaled, masked scores of rows 16 hr .. 16 hr + 15
        auto load_x = [&](float (&x)[16]) {
          uint32_t sraw[16];
          tc::tmem_ld16(tmem + lane_base + kTcColS + 32 * b + 16 * hr, sraw);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(sraw[i]) * scale;
          if (need_lim) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (pos >= sm.lim[16 * hr + i]) x[i] = -INFINITY;
          }
        };
        float x[16];
        load_x(x);
        // running maxima: every softmax warp keeps its own copy (all compute the same values)
        auto load_m = [&](float (&m)[16]) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 m4 = *reinterpret_cast<const float4*>(&sm.mrow[lq][16 * hr + i]);
            m[i] = m4.x;
            m[i + 1] = m4.y;
            m[i + 2] = m4.z;
            m[i + 3] = m4.w;
          }
        };
        float mcur[16];
        load_m(mcur);
        bool need = false;
#pragma unroll
        for (int i = 0; i < 16; ++i) need = need || (x[i] > mcur[i] + kTcHeadroom);
        float alpha_l = 1.0f;  // lane i (and i + 16): the factor of row 16 hr + i
        bool rescale = false;
        if (hr == 0 ? tc::bar_or(1, 128, need) : tc::bar_or(2, 128, need)) {
          // new row maxima over the stage's 128 tokens
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const int4 v4 = make_int4(__reduce_max_sync(0xffffffffu, tc_ord(x[i])),
                                      __reduce_max_sync(0xffffffffu, tc_ord(x[i + 1])),
                                      __reduce_max_sync(0xffffffffu, tc_ord(x[i + 2])),
                                      __reduce_max_sync(0xffffffffu, tc_ord(x[i + 3])));
            if (lane == 0) *reinterpret_cast<int4*>(&sm.red[lq][16 * hr + i]) = v4;
          }
          if (hr == 0) tc::bar_sync(1, 128); else tc::bar_sync(2, 128);
          // lane i (and i + 16) handles row 16 hr + i: its factor alpha (the O / L columns
          // fetch it by shuffle) and this warp's copy of its new maximum.  (sm.red is
          // rewritten only after the next vote, which every warp reaches after these reads.)
          {
            const int rl = 16 * hr + (lane & 15);
            const float mold = sm.mrow[lq][rl];
            int mx = sm.red[0][rl];
#pragma unroll
            for (int w = 1; w < kTcQuarters; ++w) mx = max(mx, sm.red[w][rl]);
            const float mnew = fmaxf(mold, tc_unord(mx));
            alpha_l = (mold == -INFINITY) ? 0.0f : tc_exp2(mold - mnew);
            __syncwarp();
            if (lane < 16) sm.mrow[lq][rl] = mnew;
            __syncwarp();
          }
          rescale = st > 0 && __any_sync(0xffffffffu, alpha_l != 1.0f);
          load_m(mcur);
        }
        // P^T[b] (fp16) rows 16 hr .. 16 hr + 15
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float mu0 = (mcur[i] == -INFINITY) ? 0.0f : mcur[i];
          const float mu1 = (mcur[i + 1] == -INFINITY) ? 0.0f : mcur[i + 1];
          const __half2 ph = __floats2half2_rn(tc_exp2(x[i] - mu0), tc_exp2(x[i + 1] - mu1));
          pk[i >> 1] = *reinterpret_cast<const uint32_t*>(&ph);
        }
        uint8_t* pt = sm.pt[b] + pt_off + (2 * hr) * kTcVtSbo;
        *reinterpret_cast<uint4*>(pt) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(pt + kTcVtSbo) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        if (rescale) {
          // O and L hold every PV before stage st once the PV of stage st - 1 is done;
          // this stage's P is already written, so that wait overlaps its computation.
          // The PV of stage st waits for this warp's arrival below.
          wait(b_pv + 8 * (b ^ 1), ((st - 1) >> 1) & 1);
          tc::tc_fence_after();
#pragma unroll
          for (int hh = 0; hh < 3; ++hh) {
            // O dims [0, 128), [128, 256), then L
            const uint32_t col = tmem + lane_base + (hh < 2 ? kTcColO + 32 * hh : kTcColL) + 16 * hr;
            uint32_t o[16];
            tc::tmem_ld16(col, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i)
              o[i] = __float_as_uint(__uint_as_float(o[i]) * __shfl_sync(0xffffffffu, alpha_l, i));
            tc::tmem_st16(col, o);
          }
          tc::tmem_wait_st();
        }
      }
      // S[b] is read: free it for the QK of stage st + 2; P^T[b] is written
      tc::tc_fence_before();
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(b_k + 8 * b);
        tc::mbar_arrive(b_p + 8 * b);
      }
    }

    // ---------------- epilogue: normalised partial O and LSE
    if (nst > 0) {
      wait(b_pv + 8 * ((nst - 1) & 1), ((nst - 1) >> 1) & 1);
      tc::tc_fence_after();
    }
    const int64_t pslot = p.part_begin[ri] + sp;
    const int64_t prow0 = (pslot * a.hk + h) * kTcRows;
    __half* po = reinterpret_cast<__half*>(a.part_o);
    if (active) {
      float L[16];
      {
        uint32_t lr[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) lr[i] = 0u;
        if (nst > 0) {
          tc::tmem_ld16(tmem + lane_base + kTcColL + 16 * hr, lr);
          tc::tmem_wait_ld();
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) L[i] = __uint_as_float(lr[i]);
      }
      // normalised O in fp16 (the merge reads it once; 2^-11 relative is far inside the
      // output tolerance), zero for empty rows: one fast reciprocal per row (2 ulp of fp32,
      // far below the fp16 rounding), the rows staged
      // in shared memory (the P^T buffers, free once the last PV is done) so that they
      // leave in 16-byte pieces below
      float rinv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) rinv[i] = (L[i] > 0.0f || L[i] != L[i]) ? __fdividef(1.0f, L[i]) : 0.0f;
      __half* so = reinterpret_cast<__half*>(&sm.pt[0][0]);  // [32 rows][256 dims]
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = 0u;
        if (nst > 0) {
          tc::tmem_ld16(tmem + lane_base + kTcColO + 32 * hh + 16 * hr, o);
          tc::tmem_wait_ld();
        }
        const int dim = tc_dim(128 * hh + tok);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          so[(16 * hr + i) * D + dim] = __float2half_rn(rinv[i] != 0.0f ? __uint_as_float(o[i]) * rinv[i] : 0.0f);
      }
      if (lq == 0 && lane < 16 && 16 * hr + lane < R) {
        float Li = 0.0f, mi = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (lane == i) {
            Li = L[i];
            mi = sm.mrow[lq][16 * hr + i];
          }
        a.part_lse[prow0 + 16 * hr + lane] =
            (Li > 0.0f || Li != Li) ? (mi + log2f(Li)) * 0.69314718055994531f : -INFINITY;
      }
    }
    // the staged rows r < R, 512 contiguous bytes each, by all softmax threads
    tc::bar_sync(3, 32 * kTcSmWarps);
    {
      const int st_tid = tid - kTcCompute;
      const uint4* so4 = reinterpret_cast<const uint4*>(&sm.pt[0][0]);
      for (int idx = st_tid; idx < R * (D / 8); idx += 32 * kTcSmWarps) {
        const int r = idx / (D / 8), c = idx - r * (D / 8);
        *reinterpret_cast<uint4*>(po + (prow0 + r) * D + 8 * c) = so4[idx];
      }
    }
  }

  // ---------------- teardown
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == kTcProdWarp) tc::tmem_dealloc(tmem, kTcCols);
}

// Merge of the splits (_merge_slab, slab_attention.py:156-194, joint form)
// with the causal current chunk: one warp per query row, lane l owning dims
// 8 l .. 8 l + 7, two rows per CTA, no block-wide barrier.  Launched as a
// programmatic dependent of decode_tc_kernel: its CTAs start on SMs the
// attention grid leaves free (or has left), score the current chunk while the
// attention runs, then wait for it and read the splits' LSEs and fp16
// partials (up to 24 splits in one round of 16-byte loads, later ones in
// rounds of eight).
constexpr int kTcCombineWarps = 2;  // 64 threads per CTA

template <typename T>
__global__ void __launch_bounds__(32 * kTcCombineWarps)
    tc_combine_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p) {
  // kFirst: partial rows loaded in the first round, enough for every split of a
  // history spread over the whole GPU (144 CTAs over >= 6 requests); kBatch: later rounds
  constexpr int D = 256, kMaxKeys = 32, kBatch = 8, kFirst = 24;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kTcCombineWarps + (threadIdx.x >> 5);
  const int per_req = a.hk * kTcRows;
  const int ri = gw / per_req;
  if (ri >= p.num_req) return;
  const int h = (gw - ri * per_req) / kTcRows, row = gw - ri * per_req - h * kTcRows;
  const int q_start = p.q_start[ri], qlen = p.q_len[ri], seq = p.seq[ri], prefix = p.prefix[ri];
  const int G = a.group;
  if (row >= qlen * G) return;
  const int tl = row / G;
  const int64_t qrow = (int64_t)(q_start + tl) * a.hq + (int64_t)h * G + (row - tl * G);
  const int np = (prefix > 0) ? p.splits[ri] : 0;
  const int nkeys = (a.k_new != nullptr) ? min(seq - prefix - (qlen - 1 - tl), kMaxKeys) : 0;
  const int64_t pbase = p.part_begin[ri];
  const __half* po = reinterpret_cast<const __half*>(a.part_o);
  auto prow_of = [&](int i) -> int64_t { return ((pbase + i) * a.hk + h) * kTcRows + row; };
  auto f8 = [](const uint4& u, float* f) {
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_f32(e[i]);
  };

  // current-chunk scores (natural-log units): key j on every lane after a warp sum
  const uint4 qu = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.q) + qrow * D + 8 * lane);
  float qf[8];
  f8(qu, qf);
  float kscore = -INFINITY;  // lane j holds the score of key j
  float gmax = -INFINITY;    // the row's maximum over splits and keys
  for (int j0 = 0; j0 < nkeys; j0 += 4) {
    uint4 ku[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      ku[u] = (j0 + u < nkeys) ? *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.k_new) +
                                                                ((int64_t)(q_start + j0 + u) * a.hk + h) * D + 8 * lane)
                               : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float kf[8];
      f8(ku[u], kf);
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(qf[i], kf[i], d);
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o2);
      if (lane == j0 + u && j0 + u < nkeys) kscore = d * a.scale_log2 * 0.69314718055994531f;
    }
  }
  // the current chunk's values do not depend on the attention grid: load them now
  constexpr int kPreV = 4;
  uint4 vpre[kPreV];
#pragma unroll
  for (int j = 0; j < kPreV; ++j)
    vpre[j] = (j < nkeys) ? *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.v_new) +
                                                           ((int64_t)(q_start + j) * a.hk + h) * D + 8 * lane)
                          : make_uint4(0u, 0u, 0u, 0u);

  // the partials are written by the attention grid this launch depends on
  // (programmatic dependent launch: this grid may start while that one runs)
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  // one round of loads: every split's LSE (lane i % 32) and the first
  // kFirst partial rows, then the maximum (NaN propagates) and weights
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
  float lsum = 0.0f;
  for (int i32 = 0; i32 < np; i32 += 32) {
    const int nb = min(32, np - i32);
    const float ls = (lane < nb) ? __ldcg(a.part_lse + prow_of(i32 + lane)) : -INFINITY;
    uint4 ou[kFirst];
#pragma unroll
    for (int u = 0; u < kFirst; ++u)
      ou[u] = (u < nb) ? __ldcg(reinterpret_cast<const uint4*>(po + prow_of(i32 + u) * D + 8 * lane))
                       : make_uint4(0u, 0u, 0u, 0u);
    float mx = (i32 == 0) ? kscore : -INFINITY;
    mx = nan_max(mx, ls);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) mx = nan_max(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
    if (i32 == 0) {
      // more than 32 splits: the maximum over the later passes joins below
      for (int j32 = 32; j32 < np; j32 += 32) {
        float m2 = (j32 + lane < np) ? __ldcg(a.part_lse + prow_of(j32 + lane)) : -INFINITY;
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) m2 = nan_max(m2, __shfl_xor_sync(0xffffffffu, m2, o2));
        mx = nan_max(mx, m2);
      }
      gmax = mx;
    }
    const float Mu = (gmax == -INFINITY) ? 0.0f : gmax;
    const float w = (lane < nb && ls != -INFINITY) ? expf(ls - Mu) : 0.0f;
    lsum += w;
#pragma unroll
    for (int u = 0; u < kFirst; ++u) {
      const float wu = __shfl_sync(0xffffffffu, w, u);
      if (u >= nb) break;
      const __half* hv = reinterpret_cast<const __half*>(&ou[u]);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(wu, __half2float(hv[e]), acc[e]);
    }
    for (int b0 = kFirst; b0 < nb; b0 += kBatch) {
      uint4 ob[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        ob[u] = (b0 + u < nb) ? __ldcg(reinterpret_cast<const uint4*>(po + prow_of(i32 + b0 + u) * D + 8 * lane))
                              : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const float wu = __shfl_sync(0xffffffffu, w, (b0 + u) & 31);
        if (b0 + u >= nb) break;
        const __half* hv = reinterpret_cast<const __half*>(&ob[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(wu, __half2float(hv[e]), acc[e]);
      }
    }
  }
  if (np == 0) gmax = kscore;
  float mx = gmax;
  if (np == 0) {
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) mx = nan_max(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
    gmax = mx;
  }
  const float Mu = (mx == -INFINITY) ? 0.0f : mx;
  // the row's current-chunk keys
  {
    const float wk = (lane < nkeys) ? expf(kscore - Mu) : 0.0f;
    lsum += wk;
#pragma unroll
    for (int j = 0; j < kPreV; ++j) {
      const float wj = __shfl_sync(0xffffffffu, wk, j);
      if (j >= nkeys) break;
      float vf[8];
      f8(vpre[j], vf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(wj, vf[e], acc[e]);
    }
    for (int j = kPreV; j < nkeys; ++j) {
      const float wj = __shfl_sync(0xffffffffu, wk, j);
      const uint4 vu = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.v_new) +
                                                       ((int64_t)(q_start + j) * a.hk + h) * D + 8 * lane);
      float vf[8];
      f8(vu, vf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(wj, vf[e], acc[e]);
    }
  }
#pragma unroll
  for (int o2 = 16; o2 > 0; o2 >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o2);
  const float den = (lsum > 0.0f || lsum != lsum) ? lsum : 1.0f;
  float4* dst = reinterpret_cast<float4*>(a.out + qrow * D + 8 * lane);
  const float rden = __fdividef(1.0f, den);  // one fast reciprocal (2 ulp) for the row's 8 values
  dst[0] = make_float4(acc[0] * rden, acc[1] * rden, acc[2] * rden, acc[3] * rden);
  dst[1] = make_float4(acc[4] * rden, acc[5] * rden, acc[6] * rden, acc[7] * rden);
  if (lane == 0) a.lse[qrow] = (mx == -INFINITY) ? -INFINITY : Mu + logf(den);
}

}  // namespace oscar
