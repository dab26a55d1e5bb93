// Continuation / prefill attention over paged INT2 history on the
// 5th-generation tensor cores (head dim 256): the tcgen05 + TMEM kernel for
// q-blocks of 128 query rows.
//
// Semantics are those of paged_attn_kernel (kernels/streaming_attention.py:
// 134-196 and kernels/slab_attention.py:376-476): keys p < prefix come from the
// packed cache (T(fp16(code * scale + zero))), an owner-tag hit reads the fp32
// staging rows instead (T(fp16(x))), keys p >= prefix are the current chunk;
// query i of a request sees keys [0, seq - q_len + i].  The work unit and the
// plan are the tile kernel's: (request, q-block of tpb tokens x G heads =
// <= 128 rows, kv split) x kv head, 64-key tiles.
//
// Layout: query rows on the 128 TMEM lanes (one row per thread of the softmax
// warps), so the online softmax of a row needs no cross-thread reduction.
//   TMEM columns: Q [0, 128) (bf16/fp16 pairs, the A operand of S = Q K^T),
//   S[0] [128, 192), S[1] [192, 256) (fp32 scores of a 64-key tile),
//   O [256, 512) (fp32, 256 dims).
//   S = Q K^T : M = 128 rows, N = 64 keys, K = 256 dims (16 MMAs), A from TMEM,
//               B = the K tile in shared memory (K-major).
//   O += P V  : M = 128 rows, N = 256 dims, K = 64 keys (4 MMAs), A = P (fp16,
//               shared memory, K-major), B = the V tile (fp16, MN-major).
// Warps 0-3 (softmax, lane quarter = warp): Q into TMEM once; per tile read S,
//   mask, keep a running row maximum that moves only when a score exceeds it by
//   more than 15 (log2 units; P = 2^(x - m) <= 2^15 stays in fp16 range, and O
//   is rescaled in TMEM on those tiles only), write P (fp16) to shared memory,
//   sum P (fp32) into the row's l; finally O / l and the LSE.
// Warps 4-11 (loaders): a thread fills one (key, 64-dim group) of a 64-key tile
//   per stage: INT2 codes through 4-entry value tables (PRMT look-ups), fp32
//   staged rows, or bf16/fp16 current-chunk rows.  Three tile stages.
// Warp 12: MMA issuer, in the fixed order QK(0), QK(1), then per tile PV(t) once
//   its P is written and QK(t + 2) once its tile is loaded, on suspending waits.
// With a pre-pass (kEff: ct_expand_kernel wrote every tile of the request's keys
//   once, in this layout, to the workspace) there are no loader warps: the MMA
//   issuer is warp 4, and a producer warp (warp 5) fetches each tile with two
//   32 KB bulk copies (192 threads), also on suspending waits.
// Every wait is bounded; a timeout flags the error, and the CTA drains.
//
// Dim order inside each 16-dim group (both operands of Q K^T, and the N index of
// V / O): k-positions 0..7 hold dims 0, 2, .., 14 and 8..15 dims 1, 3, .., 15
// (tc_dim), the order the PRMT look-up emits them; the epilogue maps O back.
#pragma once

#include "attention.cuh"
#include "decode_tc.cuh"

namespace oscar {

constexpr int kCtRows = 128;
constexpr int kCtKeys = kKT;  // 64 keys per tile
constexpr int kCtStages = 3;
constexpr int kCtSmWarps = 4;
constexpr int kCtLdWarps = 8;
constexpr int kCtMmaWarp = kCtSmWarps + kCtLdWarps;
constexpr int kCtThreads = 32 * (kCtMmaWarp + 1);  // 416
constexpr int kCtEffThreads = 32 * (kCtSmWarps + 2);  // pre-pass variant: softmax, MMA, producer
constexpr int kCtColQ = 0, kCtColS = 128, kCtColO = 256;
constexpr uint32_t kCtKSbo = 4096;  // K tile: bytes between 8-key groups (32 k-groups x 128 B)
constexpr uint32_t kCtVSbo = 1024;  // V tile: bytes between 8-dim groups (8 key groups x 128 B)
constexpr uint32_t kCtPSbo = 1024;  // P: bytes between 8-row groups (8 key groups x 128 B)
constexpr float kCtHeadroom = 15.0f;

struct CtSmem {
  uint8_t k[kCtStages][kCtKeys * 256 * 2];  // address(key, m) = (key/8)*4096 + (m/8)*128 + (key%8)*16 + (m%8)*2
  uint8_t v[kCtStages][kCtKeys * 256 * 2];  // address(key, n) = (n/8)*1024 + (key/8)*128 + (key%8)*16 + (n%8)*2
  uint8_t p[2][kCtRows * kCtKeys * 2];      // address(row, key) = (row/8)*1024 + (key/8)*128 + (row%8)*16 + (key%8)*2
  unsigned long long bar_full[kCtStages], bar_empty[kCtStages], bar_s[2], bar_p[2], bar_o[2], bar_end;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(CtSmem) <= 227 * 1024, "CtSmem exceeds the shared memory of a CTA");

// natural pairs W[i] = dims (2i, 2i + 1) of a 16-dim group -> the permuted order
// (0,2) (4,6) (8,10) (12,14) (1,3) (5,7) (9,11) (13,15)
OSCAR_DEVINL void ct_permute16(const uint32_t* w, uint32_t* r) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    r[c] = prmt(w[2 * c], w[2 * c + 1], 0x5410u);
    r[4 + c] = prmt(w[2 * c], w[2 * c + 1], 0x7632u);
  }
}

// One (key, 64-dim group) of a 64-key tile: the key's kind and its global loads
// (phase 1), then its K and V values in the tile layout (phase 2), so that a
// caller can wait for the destination between the two.
constexpr int kCtNone = 0, kCtInt2 = 1, kCtNew = 2, kCtStaged = 3;
struct CtItem {
  int kind;
  int64_t blk, seat, own;
  uint2 meta;        // INT2: K scale, K zero, V scale, V zero
  uint4 rk[8], rv[8];  // INT2: codes in [0]; current chunk: the raw 64-dim K and V rows
};

template <typename T>
OSCAR_DEVINL void ct_item_load(const AttnArgs& a, int req, int h, int q_start, int prefix, int pos, int live_end,
                               int g, CtItem& it) {
  constexpr int D = 256;
  it.kind = kCtNone;
  it.blk = 0;
  it.seat = -1;
  it.own = -1;
  it.meta = make_uint2(0, 0);
  if (pos >= live_end) return;
  if (pos >= prefix) {
    it.kind = kCtNew;
    const int64_t tk = (int64_t)q_start + (pos - prefix);
    const int64_t base = (tk * a.hk + h) * (int64_t)D + 64 * g;
    const uint4* kn = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.k_new) + base);
    const uint4* vn = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.v_new) + base);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      it.rk[i] = kn[i];
      it.rv[i] = vn[i];
    }
    return;
  }
  const int pg = pos / a.bs, off = pos - pg * a.bs;
  const int64_t blk = a.bt[(int64_t)req * a.bt_stride + pg];
  if (blk < 0 || blk >= a.num_blocks) {
    flag_error(2u);
    return;
  }
  it.kind = kCtInt2;
  it.blk = blk;
  const uint8_t* ks = a.kc + blk * a.ksb + off * a.kst + (int64_t)h * a.ksh;
  const uint8_t* vs = a.vc + blk * a.vsb + off * a.vst + (int64_t)h * a.vsh;
  if (a.owner != nullptr) {  // owner tag, loaded beside the codes
    // (a 32-bit remainder whenever both operands fit, as they do in practice)
    const int64_t rem = (blk <= 0xffffffffll && a.stage_rows <= 0xffffffffll)
                            ? (int64_t)((uint32_t)blk % (uint32_t)a.stage_rows)
                            : blk % a.stage_rows;
    it.seat = rem * a.bs + off;
    it.own = a.owner[it.seat];
  }
  if (((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs)) & 15) == 0) {
    it.meta = *reinterpret_cast<const uint2*>(ks);
    it.rk[0] = *reinterpret_cast<const uint4*>(ks + 32 + 16 * g);
    it.rv[0] = *reinterpret_cast<const uint4*>(vs + 16 * g);
  } else {
    // caches at an address or stride that is not 16-byte aligned: 16-bit reads
    auto w2 = [](const uint8_t* q) { return (uint32_t)ld_u16(q) | ((uint32_t)ld_u16(q + 2) << 16); };
    it.meta = make_uint2(w2(ks), w2(ks + 4));
    it.rk[0] = make_uint4(w2(ks + 32 + 16 * g), w2(ks + 36 + 16 * g), w2(ks + 40 + 16 * g), w2(ks + 44 + 16 * g));
    it.rv[0] = make_uint4(w2(vs + 16 * g), w2(vs + 4 + 16 * g), w2(vs + 8 + 16 * g), w2(vs + 12 + 16 * g));
  }
}

// phase 2: kdst / vdst point at the key's row of the K tile and V tile (shared or
// global memory; 16-dim group j = 4 g + jj goes to K chunks 2j, 2j + 1 and V chunks 2j, 2j + 1)
template <typename T>
OSCAR_DEVINL void ct_item_store(const AttnArgs& a, int h, int g, CtItem& it, uint8_t* kdst, uint8_t* vdst) {
  constexpr int D = 256;
  auto put = [&](int jj, const uint32_t* kr, const uint32_t* vr) {
    const int j = 4 * g + jj;
    *reinterpret_cast<uint4*>(kdst + (2 * j) * 128) = make_uint4(kr[0], kr[1], kr[2], kr[3]);
    *reinterpret_cast<uint4*>(kdst + (2 * j + 1) * 128) = make_uint4(kr[4], kr[5], kr[6], kr[7]);
    *reinterpret_cast<uint4*>(vdst + (2 * j) * kCtVSbo) = make_uint4(vr[0], vr[1], vr[2], vr[3]);
    *reinterpret_cast<uint4*>(vdst + (2 * j + 1) * kCtVSbo) = make_uint4(vr[4], vr[5], vr[6], vr[7]);
  };
  int kind = it.kind;
  if (kind == kCtInt2 && it.own == it.blk) kind = kCtStaged;  // the staging arena holds this position
  if (kind == kCtInt2) {
    const uint2 kl = tc_klut<T>(it.meta.x), vl = tc_vlut<T>(it.meta.y);
    const uint32_t kw[4] = {it.rk[0].x, it.rk[0].y, it.rk[0].z, it.rk[0].w};
    const uint32_t vw[4] = {it.rv[0].x, it.rv[0].y, it.rv[0].z, it.rv[0].w};
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      uint32_t kr[8], vr[8];
      tc_lut_word(kw[jj], kl.x, kl.y, kr);
      tc_lut_word(vw[jj], vl.x, vl.y, vr);
      put(jj, kr, vr);
    }
  } else if (kind == kCtNew) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const uint4 v0 = to_f16x8<T>(it.rv[2 * jj]), v1 = to_f16x8<T>(it.rv[2 * jj + 1]);
      const uint32_t kw[8] = {it.rk[2 * jj].x, it.rk[2 * jj].y, it.rk[2 * jj].z, it.rk[2 * jj].w,
                              it.rk[2 * jj + 1].x, it.rk[2 * jj + 1].y, it.rk[2 * jj + 1].z, it.rk[2 * jj + 1].w};
      const uint32_t vw[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      uint32_t kr[8], vr[8];
      ct_permute16(kw, kr);
      ct_permute16(vw, vr);
      put(jj, kr, vr);
    }
  } else if (kind == kCtNone) {
    const uint32_t z[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) put(jj, z, z);
  } else {  // staged: the fp32 rows of the seat
    const int64_t base = (it.seat * a.hk + h) * (int64_t)D + 64 * g;
#pragma unroll 1
    for (int jj = 0; jj < 4; ++jj) {
      uint32_t kr[8], vr[8];
      tc_pack_word<T, false>(a.stage_k + base + 16 * jj, true, kr);
      tc_pack_word<T, true>(a.stage_v + base + 16 * jj, true, vr);
      put(jj, kr, vr);
    }
  }
}

// Continuation pre-pass: every 64-key tile of each request's keys [0, seq) (and
// zeros past seq), per kv head, written once in the shared-memory tile layout
// (K tile 32 KB, then V tile 32 KB) to a.eff at tile p.eff_tile[request] + i, so
// that the q-block CTAs of the request fetch each tile with two bulk copies
// instead of each dequantising it.  Block = one tile x kv head, 256 threads =
// (key, 64-dim group) as in the loader warps of cont_tc_kernel.
template <typename T>
__global__ void __launch_bounds__(256) ct_expand_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p) {
  const int tile = blockIdx.x, h = blockIdx.y;
  const int ri = find_bucket(p.eff_tile, p.num_req, tile);
  const int i = tile - p.eff_tile[ri];
  const int lt = threadIdx.x;
  const int r = (lt >> 5) * 8 + ((lt & 31) & 7), g = (lt & 31) >> 3;
  const int pos = i * kCtKeys + r;
  CtItem it;
  ct_item_load<T>(a, p.req_id[ri], h, p.q_start[ri], p.prefix[ri], pos, p.seq[ri], g, it);
  uint8_t* base = a.eff + ((int64_t)tile * a.hk + h) * (2 * kCtKeys * 256 * 2);
  ct_item_store<T>(a, h, g, it, base + (r >> 3) * 4096 + (r & 7) * 16,
                   base + kCtKeys * 256 * 2 + (r >> 3) * 128 + (r & 7) * 16);
}

template <typename T, bool kEff>
__global__ void __launch_bounds__(kEff ? kCtEffThreads : kCtThreads, 1) cont_tc_kernel(const AttnArgs a, const __grid_constant__ AttnPlan p) {
  extern __shared__ __align__(1024) uint8_t ct_raw[];
  CtSmem& sm = *reinterpret_cast<CtSmem*>(ct_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int D = 256;

  const int item = blockIdx.x, h = blockIdx.y;
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
  const int ntiles = hi > lo ? (hi - lo + kCtKeys - 1) / kCtKeys : 0;

  const uint32_t b_full = smem_u32(&sm.bar_full[0]), b_empty = smem_u32(&sm.bar_empty[0]);
  const uint32_t b_s = smem_u32(&sm.bar_s[0]), b_p = smem_u32(&sm.bar_p[0]), b_o = smem_u32(&sm.bar_o[0]);
  const uint32_t b_end = smem_u32(&sm.bar_end);
  // the MMA warp: after the loader warps, or right after the softmax warps when the
  // tiles come from the pre-pass (kEff) by bulk copy
  constexpr int kMma = kEff ? kCtSmWarps : kCtMmaWarp;

  if (warp == kMma) {
    if (lane == 0) {
      for (int i = 0; i < kCtStages; ++i) {
        tc::mbar_init(b_full + 8 * i, kEff ? 1 : 32 * kCtLdWarps);
        tc::mbar_init(b_empty + 8 * i, 1);
      }
      for (int i = 0; i < 2; ++i) {
        tc::mbar_init(b_s + 8 * i, 1);
        tc::mbar_init(b_p + 8 * i, 32 * kCtSmWarps);
        tc::mbar_init(b_o + 8 * i, 1);
      }
      tc::mbar_init(b_end, 1);
      sm.abort = 0;
      tc::mbar_fence_init();
    }
    __syncwarp();
    tc::tmem_alloc(smem_u32(&sm.tmem), 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sm.tmem;

  auto give_up = [&](unsigned bit) {
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    flag_error(bit);
  };
  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (tc::mbar_wait(bar, parity)) return true;
    give_up(16u);
    return false;
  };

  if (warp < kCtSmWarps) {
    // ---- Q rows -> TMEM (row = token * G + head-in-group; rows >= nrows are zero)
    const int row = tid;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const bool live = row < nrows;
    const T* qsrc = reinterpret_cast<const T*>(a.q);
    if (live) {
      const int tl = row / G, hg = row - (row / G) * G;
      qsrc += ((int64_t)(q_start + tok0 + tl) * a.hq + (int64_t)h * G + hg) * D;
    }
    // two rounds of 128 dims (16 loads in flight per thread), 32 columns per store
#pragma unroll 1
    for (int c0 = 0; c0 < 4; c0 += 2) {
      uint4 w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = live ? *reinterpret_cast<const uint4*>(qsrc + 64 * c0 + 8 * i) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint4 w0 = w[8 * half + 2 * jj], w1 = w[8 * half + 2 * jj + 1];
          const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          ct_permute16(ww, r + 8 * jj);
        }
        tc::tmem_st32(tmem + lane_base + kCtColQ + 32 * (c0 + half), r);
      }
    }
    tc::tmem_wait_st();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();

  if (warp < kCtSmWarps) {
    // ============================ softmax + epilogue: one query row per thread
    const int row = tid;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    int lim = -1;
    if (row < nrows) lim = min(seq - qlen + tok0 + row / G + 1, hi);
    const float scale = a.scale_log2;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    const int p_off = (row >> 3) * 1024 + (row & 7) * 16;
#pragma unroll 1
    for (int t = 0; t < ntiles; ++t) {
      const int b = t & 1;
      if (!__all_sync(0xffffffffu, wait(b_s + 8 * b, (t >> 1) & 1))) { ok = false; break; }
      tc::tc_fence_after();
      uint32_t sr[64];
      tc::tmem_ld32(tmem + lane_base + kCtColS + 64 * b, sr);
      tc::tmem_ld32(tmem + lane_base + kCtColS + 64 * b + 32, sr + 32);
      tc::tmem_wait_ld();
      const int nvis = lim - (lo + t * kCtKeys);  // keys c < nvis of this tile are visible
      // row maximum of the raw scores (four independent chains; scale > 0 commutes with max);
      // masking only on tiles that reach past a row's last visible key
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (__any_sync(0xffffffffu, nvis < kCtKeys)) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float v = c < nvis ? __uint_as_float(sr[c]) : -INFINITY;
          sr[c] = __float_as_uint(v);
          m4[c & 3] = fmaxf(m4[c & 3], v);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(sr[c]));
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale;
      const bool grow = mx > m_run + kCtHeadroom;
      const bool rescale = grow && m_run != -INFINITY;
      const float alpha = rescale ? exp2f(m_run - mx) : 1.0f;
      if (grow) m_run = mx;
      if (__any_sync(0xffffffffu, rescale)) {
        // O holds tiles < t: wait for PV(t - 1) (its commit covers every earlier MMA)
        if (!__all_sync(0xffffffffu, wait(b_o + 8 * ((t - 1) & 1), ((t - 1) >> 1) & 1))) { ok = false; break; }
        tc::tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < 256; c0 += 32) {
          uint32_t o[32];
          tc::tmem_ld32(tmem + lane_base + kCtColO + c0, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tc::tmem_st32(tmem + lane_base + kCtColO + c0, o);
        }
        tc::tmem_wait_st();
        l_run *= alpha;
      }
      const float nmuse = (m_run == -INFINITY) ? 0.0f : -m_run;
      uint8_t* prow = sm.p[b] + p_off;
      // P = 2^(x scale - m) in fp16 (masked keys: 2^-inf = 0); l sums the fp32 values
      float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int kc = 0; kc < 8; ++kc) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p0 = tc_exp2(fmaf(__uint_as_float(sr[8 * kc + 2 * i]), scale, nmuse));
          const float p1 = tc_exp2(fmaf(__uint_as_float(sr[8 * kc + 2 * i + 1]), scale, nmuse));
          l4[i] += p0 + p1;
          const __half2 h2 = __floats2half2_rn(p0, p1);
          w[i] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(prow + kc * 128) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      tc::fence_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(b_p + 8 * b);
    }

    // ---- epilogue: O / l, LSE; the last PV's commit covers every MMA (waits and
    // their outcomes are warp-uniform: tcgen05.ld needs the whole warp)
    if (ok && ntiles > 0) {
      ok = __all_sync(0xffffffffu, wait(b_o + 8 * ((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1));
      tc::tc_fence_after();
    }
    if (ok) {
      const bool single = (S == 1);
      const int pslot = single ? 0 : (p.part_begin[ri] + local);
      const float den = (l_run > 0.0f || l_run != l_run) ? l_run : 1.0f;
      const float inv = 1.0f / den;
      const float lse = (m_run + log2f(den)) * 0.69314718055994531f;
      float* dst = nullptr;
      float* lse_dst = nullptr;
      if (row < nrows) {
        if (single) {
          const int tl = row / G, hg = row - (row / G) * G;
          const int64_t qrow = (int64_t)(q_start + tok0 + tl) * a.hq + (int64_t)h * G + hg;
          dst = a.out + qrow * D;
          lse_dst = a.lse + qrow;
        } else {
          const int64_t prow = ((int64_t)pslot * a.hk + h) * kCtRows + row;
          dst = a.part_o + prow * D;
          lse_dst = a.part_lse + prow;
        }
      }
#pragma unroll 1
      for (int c0 = 0; c0 < 256; c0 += 32) {
        uint32_t o[32];
        if (ntiles > 0) {
          tc::tmem_ld32(tmem + lane_base + kCtColO + c0, o);
          tc::tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (dst != nullptr) {
          // columns 16 j + i hold dim 16 j + 2 i (i < 8) and 16 j + 2 (i - 8) + 1 (i >= 8)
#pragma unroll
          for (int jj = 0; jj < 2; ++jj)
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const uint32_t* oc = o + 16 * jj;
              *reinterpret_cast<float4*>(dst + c0 + 16 * jj + 4 * q4) =
                  make_float4(__uint_as_float(oc[2 * q4]) * inv, __uint_as_float(oc[8 + 2 * q4]) * inv,
                              __uint_as_float(oc[2 * q4 + 1]) * inv, __uint_as_float(oc[9 + 2 * q4]) * inv);
            }
        }
      }
      if (lse_dst != nullptr) *lse_dst = lse;
    }
  } else if (!kEff && warp < kMma) {
    // ============================ loaders: thread = (key r, 64-dim group g) of each tile.
    // The look-ups and global loads of tile t go out before the wait for its
    // stage (PV of tile t - 3), so their latency hides behind that wait; the
    // dequantisation and the shared-memory stores follow it.
    const int lt = tid - 32 * kCtSmWarps;
    const int r = (lt >> 5) * 8 + (lane & 7), g = lane >> 3;
    const int k_off = (r >> 3) * 4096 + (r & 7) * 16;
    const int v_off = (r >> 3) * 128 + (r & 7) * 16;
#pragma unroll 1
    for (int t = 0; t < ntiles; ++t) {
      const int st = t % kCtStages;
      const int kt0 = lo + t * kCtKeys;
      CtItem it;
      ct_item_load<T>(a, req, h, q_start, prefix, kt0 + r, min(kt0 + kCtKeys, hi), g, it);
      if (t >= kCtStages && !wait(b_empty + 8 * st, ((t / kCtStages) - 1) & 1)) break;
      ct_item_store<T>(a, h, g, it, sm.k[st] + k_off, sm.v[st] + v_off);
      tc::fence_async_smem();
      tc::mbar_arrive(b_full + 8 * st);
    }
  } else if (kEff && warp == kMma + 1) {
    // ============================ producer (kEff): tile t of this CTA is pre-pass tile
    // eff_tile[request] + lo / 64 + t; its K and V tiles arrive by two bulk copies once
    // PV(t - 3) has freed stage t % 3.  One elected lane issues.
    constexpr uint32_t kTileBytes = kCtKeys * 256 * 2;
    const uint8_t* eff0 = a.eff + ((int64_t)(p.eff_tile[ri] + lo / kCtKeys) * a.hk + h) * (2 * kTileBytes);
    int rf = 0;
#pragma unroll 1
    for (; rf < ntiles; ++rf) {
      const int st = rf % kCtStages;
      // (a suspending, bounded wait: the warp takes no issue slots from the softmax warps
      // of its SM sub-partition meanwhile)
      if (rf >= kCtStages && !__all_sync(0xffffffffu, wait(b_empty + 8 * st, ((rf / kCtStages) - 1) & 1))) break;
      if (tc::elect_one()) {
        const uint8_t* src = eff0 + (int64_t)rf * a.hk * (2 * kTileBytes);
        tc::mbar_expect_tx(b_full + 8 * st, 2 * kTileBytes);
        tc::bulk_load(smem_u32(sm.k[st]), src, kTileBytes, b_full + 8 * st);
        tc::bulk_load(smem_u32(sm.v[st]), src + kTileBytes, kTileBytes, b_full + 8 * st);
      }
      __syncwarp();
    }
    // no bulk copy may still be writing shared memory when the CTA ends (abort path):
    // the last tile issued on each stage has landed
    for (int t = max(0, rf - kCtStages); t < rf; ++t)
      if (!tc::mbar_wait(b_full + 8 * (t % kCtStages), (t / kCtStages) & 1)) break;
  } else {
    // ============================ MMA issuer (one elected lane issues; the warp runs the loop)
    constexpr uint32_t idesc_qk =
        tc::instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u, 0, 0, 128, kCtKeys);
    constexpr uint32_t idesc_pv = tc::instr_desc(0u, 0, 1, 128, 256);
    // descriptors of k-step 0; k-step j starts 256 j bytes later (+16 j in the start field)
    const uint64_t dk0 = tc::smem_desc(smem_u32(sm.k[0]), 128, kCtKSbo);
    const uint64_t dv0 = tc::smem_desc(smem_u32(sm.v[0]), 128, kCtVSbo);
    const uint64_t dp0 = tc::smem_desc(smem_u32(sm.p[0]), 128, kCtPSbo);
    auto issue_qk = [&](int qs) {  // S[qs & 1] = Q K^T of tile qs
      tc::tc_fence_after();
      const uint64_t dka = dk0 + (uint64_t)((qs % kCtStages) * (sizeof(sm.k[0]) >> 4));
      const uint32_t d_s = tmem + kCtColS + 64 * (qs & 1);
      if (tc::elect_one()) {
#pragma unroll
        for (int j = 0; j < D / 16; ++j) tc::mma_ts(d_s, tmem + kCtColQ + 8 * j, dka + 16 * j, idesc_qk, j > 0 ? 1u : 0u);
        tc::mma_commit(b_s + 8 * (qs & 1));
      }
      __syncwarp();
    };
    auto issue_pv = [&](int ps) {  // O += P V of tile ps; its commits release the stage and mark O
      tc::tc_fence_after();
      const uint64_t dva = dv0 + (uint64_t)((ps % kCtStages) * (sizeof(sm.v[0]) >> 4));
      const uint64_t dpa = dp0 + (uint64_t)((ps & 1) * (sizeof(sm.p[0]) >> 4));
      if (tc::elect_one()) {
#pragma unroll
        for (int j = 0; j < kCtKeys / 16; ++j)
          tc::mma_ss(tmem + kCtColO, dpa + 16 * j, dva + 16 * j, idesc_pv, (ps > 0 || j > 0) ? 1u : 0u);
        tc::mma_commit(b_empty + 8 * (ps % kCtStages));
        tc::mma_commit(b_o + 8 * (ps & 1));
      }
      __syncwarp();
    };
    {
      // a fixed order: QK(0), QK(1), then per tile PV(t) and QK(t + 2) (S[t & 1] is free once
      // PV(t) is issued: the softmax of tile t has read it).  Suspending, bounded waits leave
      // the issue slots of this SM sub-partition to its softmax warp.
#pragma unroll 1
      for (int t = 0; t < min(2, ntiles); ++t) {
        if (!__all_sync(0xffffffffu, wait(b_full + 8 * (t % kCtStages), (t / kCtStages) & 1))) break;
        issue_qk(t);
      }
#pragma unroll 1
      for (int t = 0; t < ntiles; ++t) {
        if (*reinterpret_cast<volatile int*>(&sm.abort) != 0) break;
        if (!__all_sync(0xffffffffu, wait(b_p + 8 * (t & 1), (t >> 1) & 1))) break;
        issue_pv(t);
        const int q2 = t + 2;
        if (q2 < ntiles) {
          if (!__all_sync(0xffffffffu, wait(b_full + 8 * (q2 % kCtStages), (q2 / kCtStages) & 1))) break;
          issue_qk(q2);
        }
      }
    }
    // no MMA may be in flight when the tensor memory is freed
    if (tc::elect_one()) tc::mma_commit(b_end);
    __syncwarp();
    if (!tc::mbar_wait(b_end, 0) && lane == 0) give_up(16u);
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == kMma) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace oscar
