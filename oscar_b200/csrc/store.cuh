// K1 INT2 store and K5 staging-window kernels.
//
// K1 restates kernels/store_kernel.py:54-102 (oscar_store_ref, built on
// format.py:51-88) with the clamp of backend.py:140-146 folded in.  One warp
// owns the K or the V half of one (token, kv-head) vector; lane L owns code
// bytes L and L+32 (dims 4L..4L+3 and 4L+128..4L+131), so loads are
// float4-coalesced and each code byte is produced by exactly one lane.  All arithmetic is IEEE fp32 with
// explicit round-to-nearest intrinsics (no FMA contraction), which makes the
// codes and fp16 scale/zero bytes bit-identical to the torch CPU reference.
#pragma once

#include <climits>

#include "common.cuh"

namespace oscar {

constexpr int kMetaBytes = 8;
constexpr int kKIdxOff = 32;
constexpr float kScaleFloor = 6.103515625e-05f;  // 2^-14, format.py:38

struct StoreGeom {
  uint8_t* kc;
  uint8_t* vc;
  int64_t num_blocks;
  int block_size;
  int64_t ksb, kst, ksh;  // K cache strides in bytes
  int64_t vsb, vst, vsh;  // V cache strides in bytes
};

// k-th smallest |x| (k = clip_idx, 0-based) over the warp's vector: the
// smallest u with #{|x| <= u} > k, found two bits per step (radix 4) over the
// bit patterns (non-negative floats order like their uint32 patterns).  Step b
// keeps the largest j in 0..3 with #{|x| <= ans + j 2^b - 1} <= k; the three
// counts travel packed in one word, so a step costs one warp reduction.
template <int BPL>
OSCAR_DEVINL float kth_abs(const float (&x)[BPL][4], const bool (&act)[BPL], int k) {
  uint32_t a[BPL][4];
#pragma unroll
  for (int j = 0; j < BPL; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) a[j][e] = act[j] ? (__float_as_uint(x[j][e]) & 0x7fffffffu) : 0xffffffffu;
  uint32_t ans = 0;
#pragma unroll 1
  for (int b = 30; b >= 0; b -= 2) {
    const uint32_t p1 = ans + ((1u << b) - 1u), p2 = ans + ((2u << b) - 1u), p3 = ans + ((3u << b) - 1u);
    // the three counts (each <= 256) in 10-bit fields of one word: one warp sum per digit.
    // p1 < p2 < p3, so a value below t of them adds to the last t fields:
    // 0x100401 masked by ~0 << (30 - 10 t).  Contributions are independent and
    // summed as a tree, keeping the step's dependency chain short.
    uint32_t v[4 * BPL];
#pragma unroll
    for (int j = 0; j < BPL; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t x = a[j][e];
        const int t = (x <= p1 ? 1 : 0) + (x <= p2 ? 1 : 0) + (x <= p3 ? 1 : 0);
        v[4 * j + e] = 0x100401u & (0xffffffffu << (30 - 10 * t));
      }
#pragma unroll
    for (int w = 1; w < 4 * BPL; w <<= 1)
#pragma unroll
      for (int i = 0; i + w < 4 * BPL; i += 2 * w) v[i] += v[i + w];
    const uint32_t c = __reduce_add_sync(0xffffffffu, v[0]);
    const int c1 = (int)(c & 1023u), c2 = (int)((c >> 10) & 1023u), c3 = (int)(c >> 20);
    ans += (uint32_t)((c1 <= k ? 1 : 0) + (c2 <= k ? 1 : 0) + (c3 <= k ? 1 : 0)) << b;
  }
  return __uint_as_float(ans);
}

// The same k-th smallest |x| when it is near the top (the clip ratios in use
// keep 92-96 % of a vector, so it is the 11th or 21st largest of 256): a
// tournament over the warp.  Each lane sorts its values descending; a round
// takes the warp maximum of the lanes' heads, counts its copies (one ballot;
// a reduction only when some lane holds two) and pops them, until the count
// reaches the rank from the top.  Values order by their bit patterns, as in
// kth_abs; inactive values are 0 and can only be reached when the answer is 0.
template <int BPL>
OSCAR_DEVINL float kth_abs_top(const float (&x)[BPL][4], const bool (&act)[BPL], int rank) {
  constexpr int V = 4 * BPL;
  uint32_t a[V];
#pragma unroll
  for (int j = 0; j < BPL; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) a[4 * j + e] = act[j] ? (__float_as_uint(x[j][e]) & 0x7fffffffu) : 0u;
  // odd-even transposition sort, descending (V <= 8 values: V rounds)
#pragma unroll
  for (int r = 0; r < V; ++r)
#pragma unroll
    for (int i = r & 1; i + 1 < V; i += 2) {
      const uint32_t hi = max(a[i], a[i + 1]), lo = min(a[i], a[i + 1]);
      a[i] = hi;
      a[i + 1] = lo;
    }
  uint32_t m = 0;
  for (int round = 0; round < 32 * V; ++round) {
    m = __reduce_max_sync(0xffffffffu, a[0]);
    const bool eq0 = a[0] == m;
    const uint32_t b0 = __ballot_sync(0xffffffffu, eq0);
    const bool dup = V > 1 && __any_sync(0xffffffffu, eq0 && a[V > 1 ? 1 : 0] == m);
    int c;
    if (!dup) {
      c = __popc(b0);
    } else {
      int cl = 0;
#pragma unroll
      for (int i = 0; i < V; ++i) cl += a[i] == m ? 1 : 0;
      c = __reduce_add_sync(0xffffffffu, cl);
    }
    if (c >= rank) break;
    rank -= c;
    // pop every copy of m: one branch-free shift, more only if a lane held duplicates
#pragma unroll 1
    for (int s = 0; s < (dup ? V : 1); ++s) {
      const bool p = a[0] == m;
#pragma unroll
      for (int i = 0; i + 1 < V; ++i) a[i] = p ? a[i + 1] : a[i];
      a[V - 1] = p ? 0u : a[V - 1];
    }
  }
  return __uint_as_float(m);
}

// Quantize the warp's vector (format.quantize, format.py:67-88).
// Returns fp16 bits of scale (low 16) and zero (high 16); writes code bytes.
template <int BPL>
OSCAR_DEVINL uint32_t quantize_vec(float (&x)[BPL][4], const bool (&act)[BPL], int clip_idx,
                                   uint8_t (&code)[BPL]) {
  if (clip_idx >= 0) {
    int n_act = 0;
#pragma unroll
    for (int j = 0; j < BPL; ++j) n_act += __popc(__ballot_sync(0xffffffffu, act[j])) * 4;
    const float thr = (n_act - clip_idx <= 32) ? kth_abs_top<BPL>(x, act, n_act - clip_idx)
                                               : kth_abs<BPL>(x, act, clip_idx);
#pragma unroll
    for (int j = 0; j < BPL; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) x[j][e] = fminf(fmaxf(x[j][e], -thr), thr);
  }
  float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < BPL; ++j)
    if (act[j])
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        mn = fminf(mn, x[j][e]);
        mx = fmaxf(mx, x[j][e]);
      }
  mn = warp_min(mn);
  mx = warp_max(mx);
  float scale = __fdiv_rn(__fsub_rn(mx, mn), 3.0f);
  scale = (scale > kScaleFloor) ? scale : kScaleFloor;
  const __half sh = __float2half_rn(scale);
  const __half zh = __float2half_rn(mn);
  const float s = __half2float(sh), z = __half2float(zh);
  // q = floor(fl(fl((x - z) / s) + 0.5)) clamped to [0, 3].  The quotient
  // through the rounded reciprocal r = RN(1 / s) differs from the rounded
  // quotient by less than 2^-20 for |f| < 8, so the code only needs the
  // correctly rounded division when f lies within 2^-16 of a boundary 1, 2, 3
  // (or is not finite): that rare case takes the exact IEEE path.
  const float r = __frcp_rn(s);
#pragma unroll
  for (int j = 0; j < BPL; ++j) {
    uint32_t byte = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float dx = __fsub_rn(x[j][e], z);
      float f = __fadd_rn(__fmul_rn(dx, r), 0.5f);
      const bool near = fabsf(__fsub_rn(f, rintf(f))) <= 1.0f / 65536.0f && f > 0.5f && f < 3.5f;
      if (near || !(fabsf(f) < 8.0f)) f = __fadd_rn(__fdiv_rn(dx, s), 0.5f);
      const float q = fminf(fmaxf(floorf(f), 0.0f), 3.0f);
      byte |= ((uint32_t)(int)q & 3u) << (2 * e);
    }
    code[j] = (uint8_t)byte;
  }
  return (uint32_t)__half_as_ushort(sh) | ((uint32_t)__half_as_ushort(zh) << 16);
}

// One warp per (token, kv head, K or V): the K and V halves of a vector are
// quantized by two warps at once (warp 2 v + 0 writes the K codes and the K
// scale/zero bytes [0:4] of the K slot, warp 2 v + 1 the V codes and [4:8]).
// Warps warp0, warp0 + nwarps, ... of the task list.  `pre(tok, h, is_v, x,
// act)` runs on every task with a slot >= 0 once the row is in registers (lane
// holds floats 4 (lane + 32 j) .. + 3), before the block check and the
// quantisation: the write step stages the same row from there.
struct NoPre {
  template <int BPL>
  OSCAR_DEVINL void operator()(int64_t, int, bool, const float (&)[BPL][4], const bool (&)[BPL]) const {}
};

template <int BPL, typename Pre = NoPre>
OSCAR_DEVINL void store_tasks(int64_t warp0, int64_t nwarps, const float* __restrict__ k_rot,
                              const float* __restrict__ v_rot, int64_t n, int hk, int D, int k_clip_idx,
                              int v_clip_idx, const StoreGeom& g, const int64_t* __restrict__ slots,
                              const Pre& pre = Pre()) {
  const int NB = D / 4;  // code bytes per vector; BPL = code bytes per lane (1 or 2)
  const int lane = threadIdx.x & 31;
  const int bs_log2 = (g.block_size & (g.block_size - 1)) == 0 ? __ffs(g.block_size) - 1 : -1;
  for (int64_t task = warp0; task < 2 * n * hk; task += nwarps) {
    const int64_t vec = task >> 1;
    const bool is_v = (task & 1) != 0;
    int64_t tok;
    int h;
    if (hk == 1) {
      tok = vec;
      h = 0;
    } else if (vec < INT_MAX) {
      tok = (int)vec / hk;
      h = (int)vec - (int)tok * hk;
    } else {
      tok = vec / hk;
      h = (int)(vec - tok * hk);
    }
    const int64_t slot = slots[tok];
    if (slot < 0) continue;
    const float* src = (is_v ? v_rot : k_rot) + vec * (int64_t)D;
    float x[BPL][4];
    bool act[BPL];
#pragma unroll
    for (int j = 0; j < BPL; ++j) {
      const int b = lane + 32 * j;
      act[j] = b < NB;
      if (act[j]) {
        const float4 a = *reinterpret_cast<const float4*>(src + 4 * b);
        x[j][0] = a.x; x[j][1] = a.y; x[j][2] = a.z; x[j][3] = a.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[j][e] = 0.0f;
      }
    }
    pre(tok, h, is_v, x, act);
    int64_t blk, off;
    if (bs_log2 >= 0) {
      blk = slot >> bs_log2;
      off = slot & (g.block_size - 1);
    } else {
      blk = slot / g.block_size;
      off = slot - blk * g.block_size;
    }
    if (blk >= g.num_blocks) {
      if (lane == 0 && !is_v) flag_error(1u);
      continue;
    }
    uint8_t code[BPL];
    const uint32_t meta = quantize_vec<BPL>(x, act, is_v ? v_clip_idx : k_clip_idx, code);
    uint8_t* kslot = g.kc + blk * g.ksb + off * g.kst + (int64_t)h * g.ksh;
    uint8_t* dst = is_v ? g.vc + blk * g.vsb + off * g.vst + (int64_t)h * g.vsh : kslot + kKIdxOff;
#pragma unroll
    for (int j = 0; j < BPL; ++j) {
      const int b = lane + 32 * j;
      if (act[j]) dst[b] = code[j];
    }
    if (lane < 2) {
      // K slot bytes [0:2] K scale, [2:4] K zero, [4:6] V scale, [6:8] V zero (little endian)
      const uint16_t bits = (uint16_t)(lane ? (meta >> 16) : (meta & 0xffffu));
      uint8_t* mb = kslot + (is_v ? 4 : 0) + 2 * lane;
      mb[0] = (uint8_t)(bits & 0xffu);
      mb[1] = (uint8_t)(bits >> 8);
    }
  }
}

template <int BPL>
__global__ void __launch_bounds__(128) store_int2_kernel(const float* __restrict__ k_rot,
                                                         const float* __restrict__ v_rot, int64_t n, int hk, int D,
                                                         int k_clip_idx, int v_clip_idx, StoreGeom g,
                                                         const int64_t* __restrict__ slots) {
  pdl_release();
  pdl_wait();
  store_tasks<BPL>(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5, ((int64_t)gridDim.x * blockDim.x) >> 5,
                   k_rot, v_rot, n, hk, D, k_clip_idx, v_clip_idx, g, slots);
}

// ---------------------------------------------------------------------------
// K5 staging window

OSCAR_DEVINL int64_t staging_seat(int64_t slot, int bs, int64_t rows, int64_t* blk_out) {
  const int64_t blk = slot / bs;
  *blk_out = blk;
  return (blk % rows) * bs + (slot - blk * bs);
}

__global__ void staging_invalidate_kernel(const int64_t* __restrict__ slots, int64_t n, int64_t* __restrict__ owner,
                                          int64_t rows, int bs) {
  pdl_release();
  pdl_wait();
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    int64_t blk;
    owner[staging_seat(slot, bs, rows, &blk)] = -1;
  }
}

// pass 1: the last token (largest index) of every seat wins (stable sort +
// last-of-run in backend.py:537-544); the epoch tag makes stale entries from
// earlier calls lose without clearing the scratch.
__global__ void staging_winner_kernel(const int64_t* __restrict__ slots, int64_t n, int64_t rows, int bs,
                                      unsigned long long* __restrict__ winner, uint32_t epoch) {
  pdl_release();
  pdl_wait();
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    int64_t blk;
    const int64_t seat = staging_seat(slot, bs, rows, &blk);
    atomicMax(winner + seat, ((unsigned long long)epoch << 32) | (unsigned long long)(uint32_t)t);
  }
}

// pass 2: one warp per token; the winner writes the owner tag and, when the
// token is inside the sink/recent window, its fp32 rotated K/V (backend.py:545-555).
__global__ void __launch_bounds__(256) staging_write_kernel(
    const float* __restrict__ k_rot, const float* __restrict__ v_rot, int64_t n, int hk, int d,
    const int64_t* __restrict__ slots, const int32_t* __restrict__ qsl, const int32_t* __restrict__ seqs,
    int num_req, int sink_eff, int recent, float* __restrict__ stage_k, float* __restrict__ stage_v,
    int64_t* __restrict__ owner, int64_t rows, int bs, const unsigned long long* __restrict__ winner,
    uint32_t epoch) {
  pdl_release();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = warp; t < n; t += nwarps) {
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    int64_t blk;
    const int64_t seat = staging_seat(slot, bs, rows, &blk);
    const unsigned long long w = winner[seat];
    if ((uint32_t)(w >> 32) != epoch || (uint32_t)w != (uint32_t)t) continue;
    // request of token t: qsl[r] <= t < qsl[r+1]
    int lo = 0, hi = num_req;  // find the last r with qsl[r] <= t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (qsl[mid] <= t) lo = mid; else hi = mid;
    }
    bool keep = false;
    if (num_req > 0 && qsl[lo] <= t && t < qsl[lo + 1]) {
      const int64_t seq = seqs[lo];
      const int64_t pos = seq - qsl[lo + 1] + t;
      keep = (pos >= seq - recent) || (pos < sink_eff);
    }
    if (lane == 0) owner[seat] = keep ? blk : -1;
    if (!keep) continue;
    const int64_t row_elems = (int64_t)hk * d;
    const float4* ks = reinterpret_cast<const float4*>(k_rot + t * row_elems);
    const float4* vs = reinterpret_cast<const float4*>(v_rot + t * row_elems);
    float4* kd = reinterpret_cast<float4*>(stage_k + seat * row_elems);
    float4* vd = reinterpret_cast<float4*>(stage_v + seat * row_elems);
    for (int64_t i = lane; i < row_elems / 4; i += 32) {
      kd[i] = ks[i];
      vd[i] = vs[i];
    }
  }
}

// ---------------------------------------------------------------------------
// The write side of a decode-sized step in one launch: the INT2 store and the
// staging write (backend.py:513-555) of n <= kFusedMaxTokens tokens.  Every
// CTA loads the step's staging seats into shared memory; the warp that
// quantizes the K (or V) half of a (token, head) vector also stages that
// half: it is the seat's last writer when no later token of the step maps to
// the same seat (checked by the 32 lanes at once), the K warp of head 0 writes
// the owner tag, and a kept token's fp32 row half is copied into the arena.
// No scratch and no epoch are needed, so the launch can be replayed from a
// graph.  The owner invalidation that precedes the store in
// do_kv_cache_update (backend.py:170-176) is left out: every seat it clears
// is rewritten by that seat's last writer here.
constexpr int kFusedMaxTokens = 256;
constexpr int kFusedMaxReqs = 256;

struct StageArgs {
  const int32_t* qsl;
  const int32_t* seqs;
  int num_req, sink_eff, recent;
  float* stage_k;
  float* stage_v;
  int64_t* owner;
  int64_t rows;
  int bs;
};

template <int BPL>
__global__ void __launch_bounds__(128) write_step_kernel(const float* __restrict__ k_rot,
                                                         const float* __restrict__ v_rot, int64_t n, int hk, int D,
                                                         int k_clip_idx, int v_clip_idx, StoreGeom g,
                                                         const int64_t* __restrict__ slots, StageArgs st) {
  pdl_release();
  __shared__ int64_t s_slot[kFusedMaxTokens];
  __shared__ int s_seat[kFusedMaxTokens];  // -1: slot < 0
  __shared__ int s_qsl[kFusedMaxReqs + 1];
  __shared__ int s_seq[kFusedMaxReqs];
  const int tid = threadIdx.x, lane = tid & 31;
  const int nt = (int)n;
  // The step's slot mapping and request lists are the engine's inputs: no
  // kernel of this library writes them, so they are read while the launch in
  // front (the rotation whose rows this kernel stores) is still running; only
  // the rows wait for it.
  for (int t = tid; t < nt; t += blockDim.x) {
    const int64_t slot = slots[t];
    int64_t blk;
    s_slot[t] = slot;
    s_seat[t] = slot < 0 ? -1 : (int)staging_seat(slot, st.bs, st.rows, &blk);
  }
  for (int r = tid; r <= st.num_req; r += blockDim.x) s_qsl[r] = st.qsl[r];
  for (int r = tid; r < st.num_req; r += blockDim.x) s_seq[r] = st.seqs[r];
  __syncthreads();
  pdl_wait();

  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + tid) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  // staging, from the row the store just loaded: the seat's last writer among
  // the step's tokens (later tokens with the same seat win) writes the row if
  // its position is kept by the window, and head 0's K warp sets the owner tag
  auto stage = [&](int64_t tok64, int h, bool is_v, const float (&x)[BPL][4], const bool (&act)[BPL]) {
    const int tok = (int)tok64;
    const int seat = s_seat[tok];
    bool later = false;
    for (int u0 = tok + 1; u0 < nt; u0 += 32) {
      const int u = u0 + lane;
      later = later || (u < nt && s_seat[u] == seat);
    }
    if (__any_sync(0xffffffffu, later)) return;
    int lo = 0, hi = st.num_req;  // the last r with qsl[r] <= tok
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_qsl[mid] <= tok) lo = mid; else hi = mid;
    }
    bool keep = false;
    if (st.num_req > 0 && s_qsl[lo] <= tok && tok < s_qsl[lo + 1]) {
      const int64_t seq = s_seq[lo];
      const int64_t pos = seq - s_qsl[lo + 1] + tok;
      keep = (pos >= seq - st.recent) || (pos < st.sink_eff);
    }
    if (!is_v && h == 0 && lane == 0) st.owner[seat] = keep ? s_slot[tok] / st.bs : -1;
    if (keep) {
      float4* dst = reinterpret_cast<float4*>((is_v ? st.stage_v : st.stage_k) + ((int64_t)seat * hk + h) * D);
#pragma unroll
      for (int j = 0; j < BPL; ++j)
        if (act[j]) dst[lane + 32 * j] = make_float4(x[j][0], x[j][1], x[j][2], x[j][3]);
    }
  };
  store_tasks<BPL>(warp, nwarps, k_rot, v_rot, n, hk, D, k_clip_idx, v_clip_idx, g, s_slot, stage);
}

}  // namespace oscar
