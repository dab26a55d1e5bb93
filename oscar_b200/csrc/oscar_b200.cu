// C ABI of the B200-native OSCAR INT2 KV-cache hot path (declarations and
// contracts: include/oscar_b200.h).  One translation unit; kernels live in the
// included headers.
#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <utility>
#include <queue>
#include <vector>

#include "../../include/oscar_b200.h"
#include "attention.cuh"
#include "cont_tc.cuh"
#include "decode.cuh"
#include "decode_tc.cuh"
#include "rotate.cuh"
#include "rotate_big.cuh"
#include "rotate_tc.cuh"
#include "store.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_rotate_path{0};  // 0 auto, 1 16-row FMA tiles, 2 tensor cores, 3 128-row FMA tiles (where each applies)
std::atomic<int> g_attention_path{0};  // 0 auto, 1 tile only, 2 mma.sync decode, 3 tensor-core decode (where eligible)

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(const char* what, int launches = 1) {
  g_launches.fetch_add((uint64_t)launches, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(OSCAR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return OSCAR_OK;
}

// Launch with programmatic stream serialisation: the kernel may start while the
// previous kernel of the stream finishes; it waits (pdl_wait) before reading
// anything that kernel writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

struct DeviceInfo {
  int sms = 0;
};

DeviceInfo& device_info() {
  static thread_local int cached_dev = -1;
  static thread_local DeviceInfo info;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev);
    cached_dev = dev;
  }
  return info;
}

inline int clip_index(float ratio, int d) {
  if (!(ratio > 0.0f)) return -1;
  // backend.py:141-143: idx = min(int(ratio * D), D - 1), computed in double like Python
  const double prod = (double)ratio * (double)d;
  const int idx = (int)prod;
  return std::min(idx, d - 1);
}

}  // namespace

extern "C" {

int oscar_abi_version(void) { return 1; }

const char* oscar_last_error(void) { return g_last_error.c_str(); }

uint64_t oscar_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int oscar_set_rotation_path(int path) {
  if (path < 0 || path > 3) return fail(OSCAR_ERR_INVALID, "rotation path must be 0, 1, 2 or 3");
  g_rotate_path.store(path);
  return OSCAR_OK;
}

int oscar_set_attention_path(int path) {
  if (path < 0 || path > 3)
    return fail(OSCAR_ERR_INVALID, "attention path must be 0 (auto), 1 (tile), 2 (decode) or 3 (tensor-core decode)");
  g_attention_path.store(path);
  return OSCAR_OK;
}

int oscar_device_error(void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return -fail(OSCAR_ERR_CUDA, "stream sync failed");
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, oscar::g_bounds_error, sizeof(v)) != cudaSuccess) return -OSCAR_ERR_CUDA;
  cudaMemcpyToSymbol(oscar::g_bounds_error, &zero, sizeof(zero));
  return (int)v;
}

// ---------------------------------------------------------------------------
int oscar_store_int2(const float* k_rot, const float* v_rot, int64_t n_tokens, int32_t num_kv_heads,
                     int32_t head_dim, float k_clip_ratio, float v_clip_ratio, uint8_t* k_cache,
                     uint8_t* v_cache, int64_t num_blocks, int32_t block_size, int64_t k_stride_block,
                     int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_block,
                     int64_t v_stride_token, int64_t v_stride_head, const int64_t* slot_mapping, void* stream) {
  if (n_tokens < 0 || num_kv_heads < 1 || block_size < 1 || num_blocks < 0)
    return fail(OSCAR_ERR_INVALID, "store: invalid geometry");
  if (head_dim % 4 != 0 || head_dim / 4 > 64 || head_dim < 4)
    return fail(OSCAR_ERR_INVALID, "store: D=%d must be a multiple of 4 and at most 256", head_dim);
  if (!(k_clip_ratio >= 0.0f && k_clip_ratio <= 1.0f && v_clip_ratio >= 0.0f && v_clip_ratio <= 1.0f))
    return fail(OSCAR_ERR_INVALID, "store: clip ratios must be in [0, 1]");
  if (k_stride_head < 32 + head_dim / 4 || v_stride_head < head_dim / 4)
    return fail(OSCAR_ERR_INVALID, "store: slot of %lld/%lld bytes cannot hold the K (%d B) / V (%d B) layout",
                (long long)k_stride_head, (long long)v_stride_head, 32 + head_dim / 4, head_dim / 4);
  if (n_tokens == 0) return OSCAR_OK;
  if (!k_rot || !v_rot || !k_cache || !v_cache || !slot_mapping) return fail(OSCAR_ERR_INVALID, "store: null pointer");
  if ((reinterpret_cast<uintptr_t>(k_rot) | reinterpret_cast<uintptr_t>(v_rot)) & 15)
    return fail(OSCAR_ERR_INVALID, "store: k_rot/v_rot must be 16-byte aligned");
  oscar::StoreGeom g{k_cache, v_cache, num_blocks, block_size, k_stride_block, k_stride_token, k_stride_head,
                     v_stride_block, v_stride_token, v_stride_head};
  const int kidx = clip_index(k_clip_ratio, head_dim), vidx = clip_index(v_clip_ratio, head_dim);
  const int64_t vecs = n_tokens * num_kv_heads;
  // one warp per (vector, K or V), four per CTA (one per scheduler): the kernel is latency-bound at decode sizes
  const int64_t blocks = std::min<int64_t>((2 * vecs + 3) / 4, (int64_t)device_info().sms * 64);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = (int)std::max<int64_t>(blocks, 1);
  if (head_dim > 128)
    launch_pdl(oscar::store_int2_kernel<2>, dim3(grid), dim3(128), 0, s, k_rot, v_rot, n_tokens, num_kv_heads,
               head_dim, kidx, vidx, g, slot_mapping);
  else
    launch_pdl(oscar::store_int2_kernel<1>, dim3(grid), dim3(128), 0, s, k_rot, v_rot, n_tokens, num_kv_heads,
               head_dim, kidx, vidx, g, slot_mapping);
  return cuda_status("store_int2_kernel");
}

int oscar_write_step(const float* k_rot, const float* v_rot, int64_t n_tokens, int32_t num_kv_heads, int32_t head_dim,
                     float k_clip_ratio, float v_clip_ratio, uint8_t* k_cache, uint8_t* v_cache, int64_t num_blocks,
                     int32_t block_size, int64_t k_stride_block, int64_t k_stride_token, int64_t k_stride_head,
                     int64_t v_stride_block, int64_t v_stride_token, int64_t v_stride_head,
                     const int64_t* slot_mapping, const int32_t* qsl, const int32_t* seqs, int32_t num_requests,
                     int32_t sink_eff, int32_t recent_tokens, float* stage_k, float* stage_v, int64_t* owner,
                     int64_t stage_rows, void* stream) {
  if (n_tokens < 0 || num_kv_heads < 1 || block_size < 1 || num_blocks < 0 || stage_rows < 1 || num_requests < 0)
    return fail(OSCAR_ERR_INVALID, "write_step: invalid geometry");
  if (n_tokens > oscar::kFusedMaxTokens || num_requests > oscar::kFusedMaxReqs || stage_rows * block_size >= INT32_MAX)
    return fail(OSCAR_ERR_UNSUPPORTED, "write_step: at most %d tokens and %d requests (use oscar_store_int2 + "
                                       "oscar_staging_write)", oscar::kFusedMaxTokens, oscar::kFusedMaxReqs);
  if (head_dim % 4 != 0 || head_dim / 4 > 64 || head_dim < 4)
    return fail(OSCAR_ERR_INVALID, "store: D=%d must be a multiple of 4 and at most 256", head_dim);
  if (!(k_clip_ratio >= 0.0f && k_clip_ratio <= 1.0f && v_clip_ratio >= 0.0f && v_clip_ratio <= 1.0f))
    return fail(OSCAR_ERR_INVALID, "store: clip ratios must be in [0, 1]");
  if (k_stride_head < 32 + head_dim / 4 || v_stride_head < head_dim / 4)
    return fail(OSCAR_ERR_INVALID, "store: slot of %lld/%lld bytes cannot hold the K (%d B) / V (%d B) layout",
                (long long)k_stride_head, (long long)v_stride_head, 32 + head_dim / 4, head_dim / 4);
  if (n_tokens == 0) return OSCAR_OK;
  if (!k_rot || !v_rot || !k_cache || !v_cache || !slot_mapping || !stage_k || !stage_v || !owner ||
      (num_requests > 0 && (!qsl || !seqs)))
    return fail(OSCAR_ERR_INVALID, "write_step: null pointer");
  if ((reinterpret_cast<uintptr_t>(k_rot) | reinterpret_cast<uintptr_t>(v_rot) | reinterpret_cast<uintptr_t>(stage_k) |
       reinterpret_cast<uintptr_t>(stage_v)) & 15)
    return fail(OSCAR_ERR_INVALID, "write_step: fp32 arrays must be 16-byte aligned");
  oscar::StoreGeom g{k_cache, v_cache, num_blocks, block_size, k_stride_block, k_stride_token, k_stride_head,
                     v_stride_block, v_stride_token, v_stride_head};
  oscar::StageArgs st{qsl, seqs, num_requests, sink_eff, recent_tokens, stage_k, stage_v, owner, stage_rows,
                      block_size};
  const int kidx = clip_index(k_clip_ratio, head_dim), vidx = clip_index(v_clip_ratio, head_dim);
  const int64_t tasks = 2 * n_tokens * num_kv_heads;
  // one warp per (token, head, K or V) task, four per CTA
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((tasks + 3) / 4, (int64_t)device_info().sms * 64));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (head_dim > 128)
    launch_pdl(oscar::write_step_kernel<2>, dim3(grid), dim3(128), 0, s, k_rot, v_rot, n_tokens, num_kv_heads,
               head_dim, kidx, vidx, g, slot_mapping, st);
  else
    launch_pdl(oscar::write_step_kernel<1>, dim3(grid), dim3(128), 0, s, k_rot, v_rot, n_tokens, num_kv_heads,
               head_dim, kidx, vidx, g, slot_mapping, st);
  return cuda_status("write_step_kernel");
}

int oscar_staging_invalidate(const int64_t* slot_mapping, int64_t n_tokens, int64_t* owner, int64_t stage_rows,
                             int32_t block_size, void* stream) {
  if (n_tokens < 0 || stage_rows < 1 || block_size < 1) return fail(OSCAR_ERR_INVALID, "staging: invalid geometry");
  if (n_tokens == 0) return OSCAR_OK;
  if (!slot_mapping || !owner) return fail(OSCAR_ERR_INVALID, "staging: null pointer");
  const int grid = (int)std::min<int64_t>((n_tokens + 255) / 256, 4096);
  launch_pdl(oscar::staging_invalidate_kernel, dim3(grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
             slot_mapping, n_tokens, owner, stage_rows, block_size);
  return cuda_status("staging_invalidate_kernel");
}

int oscar_staging_write(const float* k_rot, const float* v_rot, int64_t n_tokens, int32_t num_kv_heads,
                        int32_t head_dim, const int64_t* slot_mapping, const int32_t* qsl, const int32_t* seqs,
                        int32_t num_requests, int32_t sink_eff, int32_t recent_tokens, float* stage_k,
                        float* stage_v, int64_t* owner, int64_t stage_rows, int32_t block_size,
                        uint64_t* seat_winner, uint32_t epoch, void* stream) {
  if (n_tokens < 0 || num_kv_heads < 1 || head_dim < 4 || head_dim % 4 || stage_rows < 1 || block_size < 1 ||
      num_requests < 0 || n_tokens >= (int64_t)0xffffffffLL)
    return fail(OSCAR_ERR_INVALID, "staging: invalid geometry");
  if (epoch == 0) return fail(OSCAR_ERR_INVALID, "staging: epoch must start at 1");
  if (n_tokens == 0) return OSCAR_OK;
  if (!k_rot || !v_rot || !slot_mapping || !stage_k || !stage_v || !owner || !seat_winner ||
      (num_requests > 0 && (!qsl || !seqs)))
    return fail(OSCAR_ERR_INVALID, "staging: null pointer");
  if ((reinterpret_cast<uintptr_t>(k_rot) | reinterpret_cast<uintptr_t>(v_rot) | reinterpret_cast<uintptr_t>(stage_k) |
       reinterpret_cast<uintptr_t>(stage_v)) & 15)
    return fail(OSCAR_ERR_INVALID, "staging: fp32 arrays must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid1 = (int)std::min<int64_t>((n_tokens + 255) / 256, 4096);
  launch_pdl(oscar::staging_winner_kernel, dim3(grid1), dim3(256), 0, s, slot_mapping, n_tokens, stage_rows,
             block_size, reinterpret_cast<unsigned long long*>(seat_winner), epoch);
  const int grid2 = (int)std::min<int64_t>((n_tokens + 7) / 8, (int64_t)device_info().sms * 16);
  launch_pdl(oscar::staging_write_kernel, dim3(std::max(grid2, 1)), dim3(256), 0, s, k_rot, v_rot, n_tokens,
             num_kv_heads, head_dim, slot_mapping, qsl, seqs, num_requests, sink_eff, recent_tokens, stage_k, stage_v,
             owner, stage_rows, block_size, reinterpret_cast<const unsigned long long*>(seat_winner), epoch);
  return cuda_status("staging kernels", 2);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// attention

namespace {

struct ReqInfo {
  int req, q_start, q_len, seq, prefix;
};

template <int D, typename T, int NW>
size_t attn_smem_bytes() {
  return (size_t)(16 * NW + 2 * oscar::kKT) * D * sizeof(T);
}

template <int D, typename T, int NW>
int attn_ctas_per_sm() {
  static thread_local int cached_dev = -1, cached = 1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    const size_t smem = attn_smem_bytes<D, T, NW>();
    cudaFuncSetAttribute(oscar::paged_attn_kernel<D, T, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int n = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, oscar::paged_attn_kernel<D, T, NW>, NW * 32, smem) !=
        cudaSuccess)
      n = 1;
    cached = std::max(n, 1);
    cached_dev = dev;
  }
  return cached;
}

// Host planner: q-blocks per request, then split-KV factors so that the grid
// covers about `target` CTAs with near-equal key tiles per CTA; the partial
// workspace must fit `ws_bytes` (splits shrink until it does, down to 1).
struct Planned {
  oscar::AttnPlan plan;
  int64_t part_bytes;
};

Planned plan_batch(const std::vector<ReqInfo>& reqs, size_t b0, size_t b1, int rows, int group, int hk, int d,
                   int target, int64_t ws_bytes) {
  Planned out{};
  oscar::AttnPlan& p = out.plan;
  p.num_req = (int)(b1 - b0);
  p.rows = rows;
  p.tpb = rows / group;
  int64_t work = 0;
  for (size_t i = b0; i < b1; ++i) {
    const int qb = (reqs[i].q_len + p.tpb - 1) / p.tpb;
    const int nt = std::max(1, (reqs[i].seq + oscar::kKT - 1) / oscar::kKT);
    work += (int64_t)qb * nt;
  }
  int64_t budget = std::max<int64_t>(1, (work * hk + target - 1) / std::max(target, 1));
  for (;;) {
    int items = 0, merge = 0, parts = 0;
    int64_t part_bytes = 0;
    for (size_t i = b0; i < b1; ++i) {
      const int j = (int)(i - b0);
      const ReqInfo& r = reqs[i];
      const int qb = (r.q_len + p.tpb - 1) / p.tpb;
      const int nt = std::max(1, (r.seq + oscar::kKT - 1) / oscar::kKT);
      int s = (int)std::max<int64_t>(1, (nt + budget - 1) / budget);
      int chunk_tiles = (nt + s - 1) / s;
      s = (nt + chunk_tiles - 1) / chunk_tiles;
      p.req_id[j] = r.req;
      p.q_start[j] = r.q_start;
      p.q_len[j] = r.q_len;
      p.seq[j] = r.seq;
      p.prefix[j] = r.prefix;
      p.splits[j] = s;
      p.chunk[j] = chunk_tiles * oscar::kKT;
      p.item_begin[j] = items;
      p.merge_begin[j] = merge;
      p.part_begin[j] = parts;
      items += qb * s;
      if (s > 1) {
        merge += qb;
        parts += qb * s;
        part_bytes += (int64_t)qb * s * hk * rows * (d + 1) * 4;
      }
    }
    p.item_begin[p.num_req] = items;
    p.merge_begin[p.num_req] = merge;
    p.part_begin[p.num_req] = parts;
    p.total_items = items;
    p.total_merge_rows = merge * rows;
    out.part_bytes = part_bytes;
    if (part_bytes <= ws_bytes || parts == 0) break;
    budget *= 2;
  }
  return out;
}

template <int D>
int attn_ctas_per_sm_nw(int nw) {
  if (nw == 2) return attn_ctas_per_sm<D, __nv_bfloat16, 2>();
  if (nw == 8) return attn_ctas_per_sm<D, __nv_bfloat16, 8>();
  return attn_ctas_per_sm<D, __nv_bfloat16, 4>();
}

int attn_target(int d, int nw) {
  const int sms = device_info().sms;
  if (d == 256) return sms * attn_ctas_per_sm_nw<256>(nw);
  if (d == 128) return sms * attn_ctas_per_sm_nw<128>(nw);
  return sms * attn_ctas_per_sm_nw<64>(nw);
}

// query rows per tile-kernel CTA: 32 for decode-sized blocks, 128 (eight warps) for
// continuation / prefill blocks of at least 512 rows, 64 otherwise
inline int rows_for(int max_q, int group) {
  const int64_t rows = (int64_t)max_q * group;
  if (rows <= 32 && group <= 32) return 32;
  return rows >= 512 ? 128 : 64;
}

template <int D, typename T, int NW>
int run_attention(const oscar::AttnArgs& base, const std::vector<ReqInfo>& reqs, void* workspace,
                  int64_t ws_bytes, cudaStream_t s) {
  constexpr int ROWS = 16 * NW;
  const size_t smem = attn_smem_bytes<D, T, NW>();
  attn_ctas_per_sm<D, T, NW>();  // sets the dynamic shared-memory attribute
  const int target = attn_target(D, NW);
  for (size_t b0 = 0; b0 < reqs.size(); b0 += oscar::kPlanReqs) {
    const size_t b1 = std::min(reqs.size(), b0 + (size_t)oscar::kPlanReqs);
    Planned pl = plan_batch(reqs, b0, b1, ROWS, base.group, base.hk, D, target, ws_bytes);
    oscar::AttnArgs a = base;
    if (pl.part_bytes > 0) {
      const int64_t parts = pl.plan.part_begin[pl.plan.num_req];
      a.part_o = reinterpret_cast<float*>(workspace);
      a.part_lse = a.part_o + parts * base.hk * ROWS * D;
    }
    dim3 grid(pl.plan.total_items, base.hk);
    oscar::paged_attn_kernel<D, T, NW><<<grid, NW * 32, smem, s>>>(a, pl.plan);
    int st = cuda_status("paged_attn_kernel");
    if (st) return st;
    if (pl.plan.total_merge_rows > 0) {
      dim3 mgrid(pl.plan.total_merge_rows, base.hk);
      oscar::split_combine_kernel<D><<<mgrid, D / 4, 0, s>>>(a, pl.plan);
      st = cuda_status("split_combine_kernel");
      if (st) return st;
    }
  }
  return OSCAR_OK;
}

// ---- decode / MTP path (decode.cuh): history splits, then combine with the current chunk
constexpr int kDecodeNoFit = -100;

constexpr size_t kDecodeSmem = std::max(sizeof(oscar::DecSmem), sizeof(oscar::StagedSmem));

template <typename T, int NT>
int decode_ctas_per_sm() {
  static thread_local int cached_dev = -1, cached = 1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    cudaFuncSetAttribute(oscar::decode_attn_kernel<T, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kDecodeSmem);
    int n = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, oscar::decode_attn_kernel<T, NT>, 128, kDecodeSmem) !=
        cudaSuccess)
      n = 1;
    cached = std::max(n, 1);
    cached_dev = dev;
  }
  return cached;
}

struct DecodePlanned {
  oscar::AttnPlan plan;
  int64_t part_bytes;
  bool fits;
};

// Splits of each request's history [0, prefix) into chunks of whole 64-token
// stages so that about `target` CTAs run; every split writes a partial (two
// when staging is on: the INT2 one and the staged one), so the workspace must
// hold all of them.
// Estimated makespan, in stages, of splitting each request's history into
// chunks of at most `per` stages on `target` SMs that hold one CTA each: the
// CTAs start in grid order (kv heads fastest, then the items: requests longest
// first, their splits in order) on the SM that frees first, and each takes
// `overhead` (prologue, epilogue) plus its stages.
double decode_makespan(const std::vector<ReqInfo>& reqs, size_t b0, size_t b1, int hk, int stage, int64_t per,
                       int target, double overhead) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int i = 0; i < target; ++i) free_at.push(0.0);
  double makespan = 0.0;
  for (size_t i = b0; i < b1; ++i) {
    const int ns = std::max(1, (reqs[i].prefix + stage - 1) / stage);
    int sp = (int)((ns + per - 1) / per);
    const int chunk_st = (ns + sp - 1) / sp;
    sp = (ns + chunk_st - 1) / chunk_st;
    for (int s = 0; s < sp; ++s) {
      const double len = overhead + std::min(chunk_st, ns - s * chunk_st);
      for (int h = 0; h < hk; ++h) {
        const double t = free_at.top() + len;
        free_at.pop();
        free_at.push(t);
        makespan = std::max(makespan, t);
      }
    }
  }
  return makespan;
}

// Splits of each request's history [0, prefix) into chunks of whole stages so
// that about `target` CTAs run; every split writes a partial (two when staging
// is on: the INT2 one and the staged one), so the workspace must hold all of
// them.  With `overhead` > 0 (kernels holding one CTA per SM), the chunk bound
// is the candidate with the smallest decode_makespan: equal chunks a little
// over one wave would otherwise run a second wave behind the first.
DecodePlanned plan_decode(const std::vector<ReqInfo>& reqs, size_t b0, size_t b1, int rows, int hk, int bs,
                          int target, int64_t ws_bytes, bool staged, int stage = oscar::kDecStage,
                          int max_pages = oscar::kDecMaxPages, int max_stages = 1 << 20, double overhead = 0.0) {
  DecodePlanned out{};
  oscar::AttnPlan& p = out.plan;
  p.num_req = (int)(b1 - b0);
  p.rows = rows;
  p.tpb = 0;
  const int64_t max_chunk_stages =
      std::max<int64_t>(1, std::min<int64_t>((int64_t)(max_pages - 2) * bs / stage, max_stages));
  int64_t work = 0;
  for (size_t i = b0; i < b1; ++i) work += std::max(1, (reqs[i].prefix + stage - 1) / stage);
  int64_t budget = std::max<int64_t>(1, (work * hk + target - 1) / std::max(target, 1));
  if (overhead > 0.0) {
    const int64_t base = std::min(budget, max_chunk_stages);
    const int64_t cands[] = {base, (base * 5 + 3) / 4, (base * 3 + 1) / 2, base * 2, base * 3, max_chunk_stages};
    double best = -1.0;
    for (int64_t c : cands) {
      c = std::max<int64_t>(1, std::min(c, max_chunk_stages));
      const double m = decode_makespan(reqs, b0, b1, hk, stage, c, target, overhead);
      if (best < 0.0 || m < best - 1e-9 || (m <= best + 1e-9 && c > budget)) {
        best = m;
        budget = c;
      }
    }
  }
  for (;;) {
    int items = 0;
    int64_t part_bytes = 0;
    bool all_single = true;
    const int64_t per = std::min<int64_t>(budget, max_chunk_stages);
    for (size_t i = b0; i < b1; ++i) {
      const int j = (int)(i - b0);
      const ReqInfo& r = reqs[i];
      const int ns = std::max(1, (r.prefix + stage - 1) / stage);
      int sp = (int)((ns + per - 1) / per);
      const int chunk_st = (ns + sp - 1) / sp;
      sp = (ns + chunk_st - 1) / chunk_st;
      all_single = all_single && sp == 1;
      p.req_id[j] = r.req;
      p.q_start[j] = r.q_start;
      p.q_len[j] = r.q_len;
      p.seq[j] = r.seq;
      p.prefix[j] = r.prefix;
      p.splits[j] = sp;
      p.chunk[j] = chunk_st * stage;
      p.item_begin[j] = items;
      p.part_begin[j] = items;
      p.merge_begin[j] = 0;
      items += sp;
      part_bytes += (int64_t)sp * hk * rows * (256 + 1) * 4 * (staged ? 2 : 1);
    }
    p.item_begin[p.num_req] = items;
    p.part_begin[p.num_req] = items;
    p.merge_begin[p.num_req] = 0;
    p.total_items = items;
    p.total_merge_rows = 0;
    out.part_bytes = part_bytes;
    out.fits = part_bytes <= ws_bytes;
    if (out.fits || (all_single && budget >= max_chunk_stages)) break;
    budget *= 2;
  }
  return out;
}

template <typename T, int NT>
int run_decode(const oscar::AttnArgs& base, const std::vector<ReqInfo>& reqs, void* workspace, int64_t ws_bytes,
               cudaStream_t s) {
  const int target = device_info().sms * decode_ctas_per_sm<T, NT>();
  const bool staged = base.owner != nullptr;
  // plan every batch first: fall back to the tile kernel before launching anything
  std::vector<DecodePlanned> plans;
  for (size_t b0 = 0; b0 < reqs.size(); b0 += oscar::kPlanReqs) {
    const size_t b1 = std::min(reqs.size(), b0 + (size_t)oscar::kPlanReqs);
    plans.push_back(plan_decode(reqs, b0, b1, NT * 8, base.hk, base.bs, target, ws_bytes, staged));
    if (!plans.back().fits) return kDecodeNoFit;
  }
  for (const DecodePlanned& pl : plans) {
    oscar::AttnArgs a = base;
    const int64_t parts = (int64_t)pl.plan.total_items * (staged ? 2 : 1);
    a.part_o = reinterpret_cast<float*>(workspace);
    a.part_lse = a.part_o + parts * base.hk * (NT * 8) * 256;
    const int staged_items = staged ? pl.plan.total_items : 0;
    dim3 grid(staged_items + pl.plan.total_items, base.hk);
    oscar::decode_attn_kernel<T, NT><<<grid, 128, kDecodeSmem, s>>>(a, pl.plan, staged_items);
    int st = cuda_status("decode_attn_kernel");
    if (st) return st;
    dim3 cgrid(pl.plan.num_req, base.hk * NT * 8);
    oscar::decode_combine_kernel<T><<<cgrid, 256, 0, s>>>(a, pl.plan, NT * 8, staged ? 1 : 0);
    st = cuda_status("decode_combine_kernel");
    if (st) return st;
  }
  return OSCAR_OK;
}

// The decode kernel serves D = 256 with at most 24 query rows per GQA group
// and 16-byte aligned packed caches; everything else runs the tile kernel.
bool decode_eligible(int head_dim, int max_rows, const oscar::AttnArgs& a) {
  if (head_dim != 256 || max_rows > 24) return false;
  if (a.kc == nullptr || a.vc == nullptr) return false;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.vc) | (uintptr_t)a.ksb |
                       (uintptr_t)a.kst | (uintptr_t)a.ksh | (uintptr_t)a.vsb | (uintptr_t)a.vst | (uintptr_t)a.vsh;
  if (al & 15) return false;
  if (a.ksh < 96 || a.vsh < 64) return false;
  if (a.owner != nullptr && (reinterpret_cast<uintptr_t>(a.owner) & 7)) return false;
  return true;
}

template <typename T>
int run_decode_rows(const oscar::AttnArgs& a, const std::vector<ReqInfo>& reqs, int max_rows, void* ws, int64_t wsb,
                    cudaStream_t s) {
  if (max_rows <= 8) return run_decode<T, 1>(a, reqs, ws, wsb, s);
  if (max_rows <= 16) return run_decode<T, 2>(a, reqs, ws, wsb, s);
  return run_decode<T, 3>(a, reqs, ws, wsb, s);
}

// ---- tensor-core decode path (decode_tc.cuh)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// A paged cache viewed as a 2D byte matrix [num_blocks * bs tokens, token stride]
// with boxes of `box_x` bytes x `box_y` tokens.
bool make_cache_map(CUtensorMap* map, const uint8_t* base, int64_t num_blocks, int bs, int64_t token_stride,
                    int box_x, int box_y) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)token_stride, (cuuint64_t)(num_blocks * bs)};
  const cuuint64_t strides[1] = {(cuuint64_t)token_stride};
  const cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor-core kernel needs D = 256, at most 32 query rows per GQA group,
// power-of-two block sizes, contiguous pages (block stride = bs x token stride)
// and 16-byte aligned rows, heads and owner tags; TMA coordinates are int32.
bool tc_eligible(int head_dim, int max_rows, const oscar::AttnArgs& a) {
  if (head_dim != 256 || max_rows > oscar::kTcRows || a.kc == nullptr || a.vc == nullptr) return false;
  if (a.bs < 8 || (a.bs & (a.bs - 1)) != 0) return false;
  if (a.ksb != (int64_t)a.bs * a.kst || a.vsb != (int64_t)a.bs * a.vst) return false;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.vc) | (uintptr_t)a.kst |
                       (uintptr_t)a.ksh | (uintptr_t)a.vst | (uintptr_t)a.vsh;
  if (al & 15) return false;
  if (a.owner != nullptr && ((reinterpret_cast<uintptr_t>(a.owner) | reinterpret_cast<uintptr_t>(a.stage_k) |
                              reinterpret_cast<uintptr_t>(a.stage_v)) & 15))
    return false;  // staged rows are read as float4
  if (a.ksh < 96 || a.vsh < 64 || a.ksh * (a.hk - 1) + 96 > a.kst || a.vsh * (a.hk - 1) + 64 > a.vst) return false;
  if (a.num_blocks * a.bs >= ((int64_t)1 << 31) || a.kst >= ((int64_t)1 << 31)) return false;
  if ((int64_t)(oscar::kTcMaxPages - 2) * a.bs < oscar::kTcStage) return false;
  return encode_tiled() != nullptr;
}

// per-CTA cost of the tensor-core decode kernel beyond its stages, in stages
// (prologue with the first TMA round trip, epilogue, share of the merge:
// about 5 us against about 2 us per 128-token stage, from clock64 traces)
constexpr double kTcCtaOverhead = 2.5;

template <typename T>
int run_decode_tc(const oscar::AttnArgs& base, const std::vector<ReqInfo>& reqs, void* workspace, int64_t ws_bytes,
                  cudaStream_t s) {
  static thread_local int cfg_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg_dev != dev) {
    cudaFuncSetAttribute(oscar::decode_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(oscar::TcSmem));
    cfg_dev = dev;
  }
  // one CTA per SM; the staged tokens are attended inside the kernel
  const int target = device_info().sms;
  std::vector<DecodePlanned> plans;
  for (size_t b0 = 0; b0 < reqs.size(); b0 += oscar::kPlanReqs) {
    const size_t b1 = std::min(reqs.size(), b0 + (size_t)oscar::kPlanReqs);
    plans.push_back(plan_decode(reqs, b0, b1, oscar::kTcRows, base.hk, base.bs, target, ws_bytes, false,
                                oscar::kTcStage, oscar::kTcMaxPages, oscar::kTcMaxStages, kTcCtaOverhead));
    if (!plans.back().fits) return kDecodeNoFit;
    if (plans.back().plan.total_items > 65535) return kDecodeNoFit;  // the grid's y extent holds the items
  }
  CUtensorMap tmk, tmv;
  const int box_y = std::min(base.bs, oscar::kTcStage);
  if (!make_cache_map(&tmk, base.kc, base.num_blocks, base.bs, base.kst, oscar::kTcRow, box_y) ||
      !make_cache_map(&tmv, base.vc, base.num_blocks, base.bs, base.vst, oscar::kTcRow, box_y))
    return kDecodeNoFit;
  for (const DecodePlanned& pl : plans) {
    oscar::AttnArgs a = base;
    a.part_o = reinterpret_cast<float*>(workspace);  // fp16 partials in the fp32-sized slots
    a.part_lse = a.part_o + (int64_t)pl.plan.total_items * base.hk * oscar::kTcRows * 256;
    launch_pdl(oscar::decode_tc_kernel<T>, dim3(base.hk, pl.plan.total_items), dim3(oscar::kTcThreads),
               sizeof(oscar::TcSmem), s, a, pl.plan, tmk, tmv);
    int st = cuda_status("decode_tc_kernel");
    if (st) return st;
    // the merge is a programmatic dependent of the attention grid
    const int warps = pl.plan.num_req * base.hk * oscar::kTcRows;
    launch_pdl(oscar::tc_combine_kernel<T>, dim3((warps + oscar::kTcCombineWarps - 1) / oscar::kTcCombineWarps),
               dim3(32 * oscar::kTcCombineWarps), 0, s, a, pl.plan);
    st = cuda_status("tc_combine_kernel");
    if (st) return st;
  }
  return OSCAR_OK;
}

// Continuation / prefill q-blocks of 128 rows at head dim 256 on the tensor cores
// (cont_tc.cuh): the tile kernel's plan (same q-blocks, splits and workspace),
// one CTA per SM.
template <typename T>
void set_cont_tc_smem() {
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != set_dev) {
    cudaFuncSetAttribute(oscar::cont_tc_kernel<T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(oscar::CtSmem));
    cudaFuncSetAttribute(oscar::cont_tc_kernel<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(oscar::CtSmem));
    set_dev = dev;
  }
}

// pre-pass tiles of a batch: ceil(seq / 64) per request (fills plan.eff_tile)
inline int64_t cont_tc_eff_tiles(oscar::AttnPlan& plan) {
  int64_t tiles = 0;
  for (int j = 0; j < plan.num_req; ++j) {
    plan.eff_tile[j] = (int)tiles;
    tiles += (plan.seq[j] + oscar::kCtKeys - 1) / oscar::kCtKeys;
  }
  plan.eff_tile[plan.num_req] = (int)tiles;
  return tiles;
}
constexpr int64_t kCtEffTileBytes = 2LL * oscar::kCtKeys * 256 * 2;  // K and V tiles of 64 keys x 256 dims
// the pre-pass pays when each request's tiles are read by several q-blocks (at least
// four on average); with fewer, writing and re-reading the expanded tiles costs
// more than each CTA dequantising its own
inline bool cont_tc_prepass_pays(const oscar::AttnPlan& plan) {
  int64_t qblocks = 0;
  for (int j = 0; j < plan.num_req; ++j) qblocks += (plan.item_begin[j + 1] - plan.item_begin[j]) / plan.splits[j];
  return plan.num_req > 0 && qblocks >= 4LL * plan.num_req;
}
// head dim 256, more than 32 rows per KV group: the tensor-core continuation kernel
inline bool cont_tc_route(int head_dim, int max_q, int group, int path) {
  return head_dim == 256 && rows_for(max_q, group) != 32 && (path == 0 || path == 3);
}

// Continuation / prefill q-blocks of 128 rows at head dim 256 on the tensor cores
// (cont_tc.cuh): the tile kernel's plan (same q-blocks, splits and workspace),
// one CTA per SM.  When the workspace also holds every tile of the batch's keys
// after the split partials, a pre-pass writes them once in the tile layout and
// the attention CTAs fetch them by bulk copy; otherwise each CTA dequantises its
// own tiles.
template <typename T>
int run_cont_tc(const oscar::AttnArgs& base, const std::vector<ReqInfo>& reqs, void* workspace, int64_t ws_bytes,
                cudaStream_t s) {
  constexpr int D = 256;
  constexpr size_t smem = sizeof(oscar::CtSmem);
  set_cont_tc_smem<T>();
  const int target = attn_target(D, oscar::kCtRows / 16);  // the workspace bound assumes this plan
  for (size_t b0 = 0; b0 < reqs.size(); b0 += oscar::kPlanReqs) {
    const size_t b1 = std::min(reqs.size(), b0 + (size_t)oscar::kPlanReqs);
    Planned pl = plan_batch(reqs, b0, b1, oscar::kCtRows, base.group, base.hk, D, target, ws_bytes);
    oscar::AttnArgs a = base;
    if (pl.part_bytes > 0) {
      const int64_t parts = pl.plan.part_begin[pl.plan.num_req];
      a.part_o = reinterpret_cast<float*>(workspace);
      a.part_lse = a.part_o + parts * base.hk * oscar::kCtRows * D;
    }
    const int64_t tiles = cont_tc_eff_tiles(pl.plan);
    const int64_t eff_off = (pl.part_bytes + 255) & ~(int64_t)255;
    const bool pre = tiles > 0 && tiles < INT32_MAX && workspace != nullptr && cont_tc_prepass_pays(pl.plan) &&
                     (reinterpret_cast<uintptr_t>(workspace) & 255) == 0 &&
                     eff_off + tiles * base.hk * kCtEffTileBytes <= ws_bytes;
    dim3 grid(pl.plan.total_items, base.hk);
    int st;
    if (pre) {
      a.eff = reinterpret_cast<uint8_t*>(workspace) + eff_off;
      oscar::ct_expand_kernel<T><<<dim3((unsigned)tiles, base.hk), 256, 0, s>>>(a, pl.plan);
      st = cuda_status("ct_expand_kernel");
      if (st) return st;
      oscar::cont_tc_kernel<T, true><<<grid, oscar::kCtEffThreads, smem, s>>>(a, pl.plan);
    } else {
      oscar::cont_tc_kernel<T, false><<<grid, oscar::kCtThreads, smem, s>>>(a, pl.plan);
    }
    st = cuda_status("cont_tc_kernel");
    if (st) return st;
    if (pl.plan.total_merge_rows > 0) {
      dim3 mgrid(pl.plan.total_merge_rows, base.hk);
      oscar::split_combine_kernel<D><<<mgrid, D / 4, 0, s>>>(a, pl.plan);
      st = cuda_status("split_combine_kernel");
      if (st) return st;
    }
  }
  return OSCAR_OK;
}

template <int D, typename T>
int dispatch_rows(const oscar::AttnArgs& a, const std::vector<ReqInfo>& reqs, int max_q, void* ws, int64_t wsb,
                  cudaStream_t s) {
  if (cont_tc_route(D, max_q, a.group, g_attention_path.load())) return run_cont_tc<T>(a, reqs, ws, wsb, s);
  if (rows_for(max_q, a.group) == 32) return run_attention<D, T, 2>(a, reqs, ws, wsb, s);
  if (rows_for(max_q, a.group) == 128) return run_attention<D, T, 8>(a, reqs, ws, wsb, s);
  return run_attention<D, T, 4>(a, reqs, ws, wsb, s);
}

template <int D>
int dispatch_dtype(int dtype, const oscar::AttnArgs& a, const std::vector<ReqInfo>& reqs, int max_q, void* ws,
                   int64_t wsb, cudaStream_t s) {
  const int path = g_attention_path.load();
  if (D == 256 && (path == 0 || path == 3) && tc_eligible(D, max_q * a.group, a)) {
    const int st = (dtype == OSCAR_DTYPE_BF16) ? run_decode_tc<__nv_bfloat16>(a, reqs, ws, wsb, s)
                                               : run_decode_tc<__half>(a, reqs, ws, wsb, s);
    if (st != kDecodeNoFit) return st;
  }
  if (D == 256 && (path == 0 || path == 2) && decode_eligible(D, max_q * a.group, a)) {
    const int st = (dtype == OSCAR_DTYPE_BF16) ? run_decode_rows<__nv_bfloat16>(a, reqs, max_q * a.group, ws, wsb, s)
                                               : run_decode_rows<__half>(a, reqs, max_q * a.group, ws, wsb, s);
    if (st != kDecodeNoFit) return st;
  }
  if (dtype == OSCAR_DTYPE_BF16) return dispatch_rows<D, __nv_bfloat16>(a, reqs, max_q, ws, wsb, s);
  return dispatch_rows<D, __half>(a, reqs, max_q, ws, wsb, s);
}

int collect_requests(const int32_t* qsl, const int32_t* seqs, int32_t num_requests, int64_t n_tokens, bool has_new,
                     int64_t bt_rows, int64_t bt_stride, int block_size, std::vector<ReqInfo>& reqs, int& max_q,
                     bool& any_history) {
  if (num_requests < 0 || !qsl || (num_requests > 0 && !seqs)) return fail(OSCAR_ERR_INVALID, "Invalid slab query layout");
  if (qsl[0] != 0 || qsl[num_requests] != n_tokens) return fail(OSCAR_ERR_INVALID, "Invalid slab query layout");
  if (bt_rows < num_requests) return fail(OSCAR_ERR_INVALID, "Missing request block-table rows");
  max_q = 0;
  any_history = false;
  for (int r = 0; r < num_requests; ++r) {
    const int a = qsl[r], b = qsl[r + 1], seq = seqs[r];
    if (a > b || seq < 0 || (has_new && seq < b - a))
      return fail(OSCAR_ERR_INVALID, "Sequence length must cover its query chunk");
    const int prefix = has_new ? seq - (b - a) : seq;
    if (b > a && (int64_t)((prefix + block_size - 1) / block_size) > bt_stride)
      return fail(OSCAR_ERR_INVALID, "Block table cannot cover the history");
    if (b > a) {
      reqs.push_back(ReqInfo{r, a, b - a, seq, prefix});
      max_q = std::max(max_q, b - a);
      any_history = any_history || prefix > 0;
    }
  }
  // longest first: the planners lay CTAs out in request order and the hardware starts
  // them in that order, so the heaviest requests start first and short ones fill the
  // tail (a request's own plan and splits do not depend on its place)
  std::stable_sort(reqs.begin(), reqs.end(), [](const ReqInfo& x, const ReqInfo& y) { return x.seq > y.seq; });
  return OSCAR_OK;
}

}  // namespace

// The body of oscar_slab_attention and oscar_slab_attention_shard.  A history
// shard has no current chunk and every key of [0, seqs[r]) visible to every
// query row: its plan carries seq = prefix + q_len (the causal limit
// seq - q_len + t + 1 never falls below the prefix) and it runs on the decode
// kernels, which read history only below the prefix and chunk keys only from
// k_new.
static int slab_attention_impl(const void* q, const void* k_new, const void* v_new, int32_t dtype, int64_t n_tokens,
                               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, const uint8_t* k_cache,
                               const uint8_t* v_cache, int64_t num_blocks, int32_t block_size, int64_t k_stride_block,
                               int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_block,
                               int64_t v_stride_token, int64_t v_stride_head, const int32_t* block_table,
                               int64_t bt_rows, int64_t bt_stride, const int32_t* qsl, const int32_t* seqs,
                               int32_t num_requests, float scale, const float* stage_k, const float* stage_v,
                               const int64_t* owner, int64_t stage_rows, float* out, float* lse, void* workspace,
                               int64_t workspace_bytes, void* stream, bool shard) {
  if (num_q_heads < 1 || num_kv_heads < 1 || num_q_heads % num_kv_heads || n_tokens < 0 || block_size < 1)
    return fail(OSCAR_ERR_INVALID, "Invalid slab query layout");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(OSCAR_ERR_INVALID, "Both new K and V must be supplied together");
  if (dtype != OSCAR_DTYPE_BF16 && dtype != OSCAR_DTYPE_F16)
    return fail(OSCAR_ERR_UNSUPPORTED, "query dtype must be bf16 or fp16");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(OSCAR_ERR_UNSUPPORTED, "head_dim %d: kernels exist for 64, 128, 256", head_dim);
  const int group = num_q_heads / num_kv_heads;
  if (group > 64) return fail(OSCAR_ERR_UNSUPPORTED, "GQA group %d > 64", group);
  if ((stage_k == nullptr) != (owner == nullptr) || (stage_v == nullptr) != (owner == nullptr) ||
      (owner != nullptr && stage_rows < 1))
    return fail(OSCAR_ERR_INVALID, "Invalid streaming staging geometry");
  const bool has_new = k_new != nullptr;
  std::vector<ReqInfo> reqs;
  int max_q = 0;
  bool any_history = false;
  int st = collect_requests(qsl, seqs, num_requests, n_tokens, has_new, bt_rows, bt_stride, block_size, reqs, max_q,
                            any_history);
  if (st) return st;
  if (shard) {
    if (head_dim != 256 || max_q * group > oscar::kTcRows)
      return fail(OSCAR_ERR_UNSUPPORTED, "history shards run the decode kernels: head_dim 256 and at most %d query "
                  "rows per KV group", oscar::kTcRows);
    for (ReqInfo& r : reqs) r.seq = r.prefix + r.q_len;
  }
  if (any_history) {
    if (!k_cache || !v_cache || !block_table) return fail(OSCAR_ERR_INVALID, "history requires caches and a block table");
    if (k_stride_head < 32 + head_dim / 4 || v_stride_head < head_dim / 4)
      return fail(OSCAR_ERR_INVALID, "cache slot too small for the packed layout");
  }
  if (!out || !lse || (n_tokens > 0 && !q)) return fail(OSCAR_ERR_INVALID, "null output or query");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(stage_k) | reinterpret_cast<uintptr_t>(stage_v) |
       reinterpret_cast<uintptr_t>(workspace)) & 15)
    return fail(OSCAR_ERR_INVALID, "tensors must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Every query row belongs to exactly one active request (qsl covers
  // [0, n_tokens)), and every q-block writes all of its rows, so out/lse need
  // no initialisation.
  if (n_tokens == 0) return OSCAR_OK;
  oscar::AttnArgs a{};
  a.q = q;
  a.k_new = k_new;
  a.v_new = v_new;
  a.hq = num_q_heads;
  a.hk = num_kv_heads;
  a.group = group;
  a.kc = k_cache;
  a.vc = v_cache;
  a.num_blocks = num_blocks;
  a.bs = block_size;
  a.ksb = k_stride_block;
  a.kst = k_stride_token;
  a.ksh = k_stride_head;
  a.vsb = v_stride_block;
  a.vst = v_stride_token;
  a.vsh = v_stride_head;
  a.bt = block_table;
  a.bt_stride = bt_stride;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.stage_k = stage_k;
  a.stage_v = stage_v;
  a.owner = owner;
  a.stage_rows = owner ? stage_rows : 1;
  a.out = out;
  a.lse = lse;
  if (reqs.empty()) return OSCAR_OK;
  if (shard) {
    const bool bf = dtype == OSCAR_DTYPE_BF16;
    // family selector: 2 keeps the shard on the mma.sync decode kernel
    if (g_attention_path.load() != 2 && tc_eligible(256, max_q * group, a)) {
      st = bf ? run_decode_tc<__nv_bfloat16>(a, reqs, workspace, workspace_bytes, s)
              : run_decode_tc<__half>(a, reqs, workspace, workspace_bytes, s);
      if (st != kDecodeNoFit) return st;
    }
    if (decode_eligible(256, max_q * group, a)) {
      st = bf ? run_decode_rows<__nv_bfloat16>(a, reqs, max_q * group, workspace, workspace_bytes, s)
              : run_decode_rows<__half>(a, reqs, max_q * group, workspace, workspace_bytes, s);
      if (st != kDecodeNoFit) return st;
    }
    return fail(OSCAR_ERR_UNSUPPORTED, "history shard: the decode kernels do not fit this layout");
  }
  if (head_dim == 256) return dispatch_dtype<256>(dtype, a, reqs, max_q, workspace, workspace_bytes, s);
  if (head_dim == 128) return dispatch_dtype<128>(dtype, a, reqs, max_q, workspace, workspace_bytes, s);
  return dispatch_dtype<64>(dtype, a, reqs, max_q, workspace, workspace_bytes, s);
}

extern "C" {

int oscar_slab_attention(const void* q, const void* k_new, const void* v_new, int32_t dtype, int64_t n_tokens,
                         int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, const uint8_t* k_cache,
                         const uint8_t* v_cache, int64_t num_blocks, int32_t block_size, int64_t k_stride_block,
                         int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_block,
                         int64_t v_stride_token, int64_t v_stride_head, const int32_t* block_table, int64_t bt_rows,
                         int64_t bt_stride, const int32_t* qsl, const int32_t* seqs, int32_t num_requests,
                         float scale, const float* stage_k, const float* stage_v, const int64_t* owner,
                         int64_t stage_rows, float* out, float* lse, void* workspace, int64_t workspace_bytes,
                         void* stream) {
  return slab_attention_impl(q, k_new, v_new, dtype, n_tokens, num_q_heads, num_kv_heads, head_dim, k_cache, v_cache,
                             num_blocks, block_size, k_stride_block, k_stride_token, k_stride_head, v_stride_block,
                             v_stride_token, v_stride_head, block_table, bt_rows, bt_stride, qsl, seqs, num_requests,
                             scale, stage_k, stage_v, owner, stage_rows, out, lse, workspace, workspace_bytes, stream,
                             false);
}

int oscar_slab_attention_shard(const void* q, int32_t dtype, int64_t n_tokens, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, const uint8_t* k_cache, const uint8_t* v_cache,
                               int64_t num_blocks, int32_t block_size, int64_t k_stride_block, int64_t k_stride_token,
                               int64_t k_stride_head, int64_t v_stride_block, int64_t v_stride_token,
                               int64_t v_stride_head, const int32_t* block_table, int64_t bt_rows, int64_t bt_stride,
                               const int32_t* qsl, const int32_t* history_lens, int32_t num_requests, float scale,
                               const float* stage_k, const float* stage_v, const int64_t* owner, int64_t stage_rows,
                               float* out, float* lse, void* workspace, int64_t workspace_bytes, void* stream) {
  return slab_attention_impl(q, nullptr, nullptr, dtype, n_tokens, num_q_heads, num_kv_heads, head_dim, k_cache,
                             v_cache, num_blocks, block_size, k_stride_block, k_stride_token, k_stride_head,
                             v_stride_block, v_stride_token, v_stride_head, block_table, bt_rows, bt_stride, qsl,
                             history_lens, num_requests, scale, stage_k, stage_v, owner, stage_rows, out, lse,
                             workspace, workspace_bytes, stream, true);
}

int64_t oscar_slab_attention_workspace(const int32_t* qsl, const int32_t* seqs, int32_t num_requests, int32_t has_new,
                                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim) {
  if (num_q_heads < 1 || num_kv_heads < 1 || num_q_heads % num_kv_heads || num_requests < 0 || !qsl) return -1;
  std::vector<ReqInfo> reqs;
  int max_q = 0;
  bool hist = false;
  const int64_t n = qsl[num_requests];
  if (collect_requests(qsl, seqs, num_requests, n, has_new != 0, num_requests, INT32_MAX, 1, reqs, max_q, hist))
    return -1;
  const int group = num_q_heads / num_kv_heads;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return -1;
  // the path is chosen at launch from the cache layout: size for every candidate
  const int path = g_attention_path.load();
  int64_t worst = 0;
  if (head_dim == 256 && max_q * group <= oscar::kTcRows && (path == 0 || path == 3)) {
    for (size_t b0 = 0; b0 < reqs.size(); b0 += oscar::kPlanReqs) {
      const size_t b1 = std::min(reqs.size(), b0 + (size_t)oscar::kPlanReqs);
      DecodePlanned pl = plan_decode(reqs, b0, b1, oscar::kTcRows, num_kv_heads, 1 << 20, device_info().sms,
                                     INT64_MAX, false, oscar::kTcStage, oscar::kTcMaxPages, oscar::kTcMaxStages);
      worst = std::max(worst, pl.part_bytes);
    }
  }
  if (head_dim == 256 && max_q * group <= 24 && (path == 0 || path == 2)) {
    const int nt = (max_q * group + 7) / 8;
    const int per_sm = nt == 1 ? decode_ctas_per_sm<__nv_bfloat16, 1>()
                       : nt == 2 ? decode_ctas_per_sm<__nv_bfloat16, 2>()
                                 : decode_ctas_per_sm<__nv_bfloat16, 3>();
    const int target = device_info().sms * per_sm;
    for (size_t b0 = 0; b0 < reqs.size(); b0 += oscar::kPlanReqs) {
      const size_t b1 = std::min(reqs.size(), b0 + (size_t)oscar::kPlanReqs);
      // staging may be on: count the staged partials too
      DecodePlanned pl = plan_decode(reqs, b0, b1, nt * 8, num_kv_heads, 1 << 20, target, INT64_MAX, true);
      worst = std::max(worst, pl.part_bytes);
    }
  }
  const bool ct = cont_tc_route(head_dim, max_q, group, path);
  const int rows = ct ? oscar::kCtRows : rows_for(max_q, group);
  const int target = attn_target(head_dim, rows / 16);
  for (size_t b0 = 0; b0 < reqs.size(); b0 += oscar::kPlanReqs) {
    const size_t b1 = std::min(reqs.size(), b0 + (size_t)oscar::kPlanReqs);
    Planned pl = plan_batch(reqs, b0, b1, rows, group, num_kv_heads, head_dim, target, INT64_MAX);
    int64_t need = pl.part_bytes;
    if (ct && cont_tc_prepass_pays(pl.plan)) {
      // the tensor-core continuation kernel's pre-pass tiles follow the partials
      const int64_t tiles = cont_tc_eff_tiles(pl.plan);
      if (tiles > 0 && tiles < INT32_MAX) need = ((need + 255) & ~(int64_t)255) + tiles * num_kv_heads * kCtEffTileBytes;
    }
    worst = std::max(worst, need);
  }
  return worst;
}

// ---------------------------------------------------------------------------
int oscar_merge_slab(float* out, float* lse, int64_t out_rows, const void* part, int32_t part_dtype,
                     const float* part_lse, int64_t n, int32_t num_q_heads, int32_t head_dim, int64_t query_start,
                     const int32_t* query_ids, void* stream) {
  if (n < 0 || num_q_heads < 1 || head_dim < 1 || query_start < 0 || out_rows < 0)
    return fail(OSCAR_ERR_INVALID, "merge: invalid geometry");
  if (query_ids == nullptr && query_start + n > out_rows)
    return fail(OSCAR_ERR_INVALID, "merge: rows [%lld, %lld) exceed the %lld output rows", (long long)query_start,
                (long long)(query_start + n), (long long)out_rows);
  if (n == 0) return OSCAR_OK;
  if (!out || !lse || !part || !part_lse) return fail(OSCAR_ERR_INVALID, "merge: null pointer");
  const int64_t warps = n * num_q_heads;
  const int grid = (int)((warps * 32 + 255) / 256);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (part_dtype) {
    case OSCAR_DTYPE_F32:
      oscar::merge_slab_kernel<float><<<grid, 256, 0, s>>>(out, lse, out_rows, reinterpret_cast<const float*>(part), part_lse,
                                                             n, num_q_heads, head_dim, query_start, query_ids);
      break;
    case OSCAR_DTYPE_F16:
      oscar::merge_slab_kernel<__half><<<grid, 256, 0, s>>>(out, lse, out_rows, reinterpret_cast<const __half*>(part), part_lse,
                                                              n, num_q_heads, head_dim, query_start, query_ids);
      break;
    case OSCAR_DTYPE_BF16:
      oscar::merge_slab_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          out, lse, out_rows, reinterpret_cast<const __nv_bfloat16*>(part), part_lse, n, num_q_heads, head_dim, query_start,
          query_ids);
      break;
    default:
      return fail(OSCAR_ERR_INVALID, "merge: unknown part dtype");
  }
  return cuda_status("merge_slab_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Staging-window write without caller-provided scratch.
//
// Some callers of this library cannot allocate device memory at the point
// where the staging write runs (an engine whose memory planner has already
// handed every byte to the KV cache, or a plugin host that forbids cudaMalloc
// outside start-up).  For them the seat-winner scratch lives in the static
// device array below, sized for kNoAllocMaxSeats staging seats; every GPU
// that loads this library holds it (512 KiB) until the process exits.

static constexpr int64_t kNoAllocMaxSeats = 65536;
static __device__ __align__(256) unsigned long long oscar_noalloc_seat_winner[kNoAllocMaxSeats];

#include <mutex>

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[256] = {};  // device address of the array, per device ordinal

// Once per device, with that device current: the device address of the
// array.  The host symbol itself is only a host-side stand-in.
int noalloc_scratch(unsigned long long** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256)
    return fail(OSCAR_ERR_CUDA, "staging (no-alloc): no current CUDA device");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, oscar_noalloc_seat_winner);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(OSCAR_ERR_CUDA, "staging (no-alloc): cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = reinterpret_cast<unsigned long long*>(g_noalloc_ptr[dev]);
  return OSCAR_OK;
}
}  // namespace

extern "C" {

int oscar_staging_write_noalloc(const float* k_rot, const float* v_rot, int64_t n_tokens, int32_t num_kv_heads,
                                int32_t head_dim, const int64_t* slot_mapping, const int32_t* qsl,
                                const int32_t* seqs, int32_t num_requests, int32_t sink_eff, int32_t recent_tokens,
                                float* stage_k, float* stage_v, int64_t* owner, int64_t stage_rows,
                                int32_t block_size, void* stream) {
  if (n_tokens < 0 || num_kv_heads < 1 || head_dim < 4 || head_dim % 4 || stage_rows < 1 || block_size < 1 ||
      num_requests < 0 || n_tokens >= (int64_t)0xffffffffLL)
    return fail(OSCAR_ERR_INVALID, "staging (no-alloc): invalid geometry");
  if (stage_rows > kNoAllocMaxSeats / block_size)
    return fail(OSCAR_ERR_INVALID,
                "staging (no-alloc): %lld rows x %d block size = %lld seats exceed the built-in scratch of %lld "
                "seats; use oscar_staging_write with caller-provided scratch",
                (long long)stage_rows, block_size, (long long)stage_rows * block_size, (long long)kNoAllocMaxSeats);
  if (n_tokens == 0) return OSCAR_OK;
  if (!k_rot || !v_rot || !slot_mapping || !stage_k || !stage_v || !owner || (num_requests > 0 && (!qsl || !seqs)))
    return fail(OSCAR_ERR_INVALID, "staging (no-alloc): null pointer");
  if ((reinterpret_cast<uintptr_t>(k_rot) | reinterpret_cast<uintptr_t>(v_rot) | reinterpret_cast<uintptr_t>(stage_k) |
       reinterpret_cast<uintptr_t>(stage_v)) & 15)
    return fail(OSCAR_ERR_INVALID, "staging (no-alloc): fp32 arrays must be 16-byte aligned");
  unsigned long long* winner = nullptr;
  int st = noalloc_scratch(&winner);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t seats = stage_rows * block_size;
  // The array keeps the previous call's winners; they would outrank this
  // call's lower token indices, so the seats in use start from zero.
  if (cudaMemsetAsync(winner, 0, (size_t)seats * sizeof(unsigned long long), s) != cudaSuccess)
    return fail(OSCAR_ERR_CUDA, "staging (no-alloc): clearing the scratch failed");
  const uint32_t epoch = 1;
  const int grid1 = (int)std::min<int64_t>((n_tokens + 255) / 256, 4096);
  launch_pdl(oscar::staging_winner_kernel, dim3(grid1), dim3(256), 0, s, slot_mapping, n_tokens, stage_rows,
             block_size, winner, epoch);
  const int grid2 = (int)std::min<int64_t>((n_tokens + 7) / 8, (int64_t)device_info().sms * 16);
  launch_pdl(oscar::staging_write_kernel, dim3(std::max(grid2, 1)), dim3(256), 0, s, k_rot, v_rot, n_tokens,
             num_kv_heads, head_dim, slot_mapping, qsl, seqs, num_requests, sink_eff, recent_tokens, stage_k, stage_v,
             owner, stage_rows, block_size, const_cast<const unsigned long long*>(winner), epoch);
  return cuda_status("staging kernels (no-alloc)", 2);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// per-layer rotation of head vectors (backend.py:238-246 applies it with
// library GEMMs); no counterpart entry point in the reference's kernel API
namespace {

template <typename InT, typename OutT, int D>
int launch_rotate_d(const oscar::RotBatch& b, cudaStream_t s) {
  constexpr size_t smem = oscar::rotate_smem_bytes<D>();
  static thread_local int cfg_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg_dev != dev) {
    cudaFuncSetAttribute(oscar::rotate_rows_kernel<InT, OutT, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    cfg_dev = dev;
  }
  dim3 grid((unsigned)b.tile_begin[b.n], (unsigned)(D / oscar::kRotCols));
  launch_pdl(oscar::rotate_rows_kernel<InT, OutT, D>, grid, dim3(256), smem, s, b);
  return cuda_status("rotate_rows_kernel");
}

// tcgen05 (kind::tf32, split precision) rotation of a batch, in 128-row tiles
template <typename InT, typename OutT, int D>
int launch_rotate_tc_d(const oscar::RotBatch& b16, cudaStream_t s) {
  oscar::RotBatch b = b16;
  int64_t tiles = 0;
  for (int i = 0; i < b.n; ++i) {
    b.tile_begin[i] = (int)tiles;
    tiles += (b.seg[i].rows + oscar::kRtRows - 1) / oscar::kRtRows;
  }
  b.tile_begin[b.n] = (int)tiles;
  constexpr size_t smem = sizeof(oscar::RtSmem<D>);
  static thread_local int cfg_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg_dev != dev) {
    cudaFuncSetAttribute(oscar::rotate_tc_kernel<InT, OutT, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    cfg_dev = dev;
  }
  // persistent CTAs, one per SM: each column block gets SMs / blocks of them
  constexpr int kBlocks = D / oscar::kRtCols;
  const int per_block = std::max(1, device_info().sms / kBlocks);
  dim3 grid((unsigned)std::min<int64_t>(tiles, per_block), (unsigned)kBlocks);
  launch_pdl(oscar::rotate_tc_kernel<InT, OutT, D>, grid, dim3(oscar::kRtThreads), smem, s, b);
  return cuda_status("rotate_tc_kernel");
}

// automatic thresholds (rows of one segment): the tensor-core kernel from 2560
// fp32 rows (D 256: 22 us from 2048 to 3840 rows, where the 16-row tiles take
// 18 to 31 us); the register-tiled FMA kernel in 64-row tiles from 6144 rows and
// in 128-row tiles from 16384 rows.  A 64 x 128 tile takes about 27 us on its
// SM, so below 6144 rows (D 256) the 16-row tiles finish first; a smaller
// segment in 128-row tiles leaves SMs idle.
constexpr int64_t kRotTcMinRows = 2560;
constexpr int64_t kRotMidMinRows = 6144;
constexpr int64_t kRotBigMinRows = 16384;

// The tensor-core and the register-tiled kernels write 16-byte pieces of every
// output row: rows (and their starts) must be 16-byte aligned.
bool rotate_rows_aligned(const oscar::RotSeg& g, size_t out_es) {
  if (g.out != nullptr && ((reinterpret_cast<uintptr_t>(g.out) & 15) || (g.out_stride * (int64_t)out_es) % 16))
    return false;
  return g.out_f32 == nullptr || !((reinterpret_cast<uintptr_t>(g.out_f32) & 15) || g.out_f32_stride % 4);
}

// register-tiled FMA rotation of a batch, in ROWS-row tiles (D = 128 or 256)
template <typename InT, typename OutT, int D, int ROWS>
int launch_rotate_big_d(const oscar::RotBatch& b16, cudaStream_t s) {
  oscar::RotBatch b = b16;
  int64_t tiles = 0;
  for (int i = 0; i < b.n; ++i) {
    b.tile_begin[i] = (int)tiles;
    tiles += (b.seg[i].rows + ROWS - 1) / ROWS;
  }
  b.tile_begin[b.n] = (int)tiles;
  constexpr size_t smem = sizeof(oscar::RbSmem<ROWS>);
  static thread_local int cfg_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg_dev != dev) {
    cudaFuncSetAttribute(oscar::rotate_big_kernel<InT, OutT, D, ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    cfg_dev = dev;
  }
  dim3 grid((unsigned)tiles, (unsigned)(D / oscar::kRbCols));
  launch_pdl(oscar::rotate_big_kernel<InT, OutT, D, ROWS>, grid, dim3(oscar::kRbThreads), smem, s, b);
  return cuda_status("rotate_big_kernel");
}

template <typename InT, typename OutT>
int launch_rotate_fma(const oscar::RotBatch& b, int d, cudaStream_t s) {
  if (d == 256) return launch_rotate_d<InT, OutT, 256>(b, s);
  if (d == 128) return launch_rotate_d<InT, OutT, 128>(b, s);
  return launch_rotate_d<InT, OutT, 64>(b, s);
}
template <typename InT, typename OutT>
int launch_rotate_tc(const oscar::RotBatch& b, int d, cudaStream_t s) {
  if (d == 256) return launch_rotate_tc_d<InT, OutT, 256>(b, s);
  if (d == 128) return launch_rotate_tc_d<InT, OutT, 128>(b, s);
  return launch_rotate_tc_d<InT, OutT, 64>(b, s);
}

// the segments of b that `keep` selects, re-tiled in 16-row tiles
template <typename Pred>
oscar::RotBatch rotate_subset(const oscar::RotBatch& b, Pred keep) {
  oscar::RotBatch o{};
  o.rot_early = b.rot_early;
  int64_t tiles = 0;
  for (int i = 0; i < b.n; ++i) {
    if (!keep(i)) continue;
    o.seg[o.n] = b.seg[i];
    o.tile_begin[o.n] = (int)tiles;
    tiles += (b.seg[i].rows + oscar::kRotRows - 1) / oscar::kRotRows;
    ++o.n;
  }
  o.tile_begin[o.n] = (int)tiles;
  return o;
}

// Kernel of each segment, by its own size (so that a tensor is rotated the
// same way whatever it is batched with).  Automatic choice for large
// segments: the tensor cores for fp32 rows (the attention output's o @ R_v^T,
// rounded once more to the output dtype), the register-tiled FMA kernel for
// the k / v / q rotations: a k or v element on an
// INT2 quantisation boundary, or a q element on a bf16 rounding boundary next
// to an outlier channel, turns a rotation error of a few fp32 ulps into a
// visible change of the attention, and the tf32 split's error is several
// times an fp32 FMA chain's.  Smaller segments take rotate.cuh's 16-row tiles.
enum RotKernel { kRotSmall = 0, kRotBig = 1, kRotTc = 2, kRotMid = 3 };
template <typename InT>
RotKernel rotate_kernel_of(const oscar::RotSeg& g, int d, size_t out_es, int path) {
  const bool aligned = rotate_rows_aligned(g, out_es);
  if (path == 1 || !aligned) return kRotSmall;
  if (path == 2) return kRotTc;
  const RotKernel tiled = g.rows >= kRotBigMinRows ? kRotBig : kRotMid;
  if (path == 3) return d >= oscar::kRbCols ? tiled : kRotSmall;
  if (std::is_same<InT, float>::value) return g.rows >= kRotTcMinRows ? kRotTc : kRotSmall;
  return (g.rows >= kRotMidMinRows && d >= oscar::kRbCols) ? tiled : kRotSmall;
}

template <typename InT, typename OutT>
int launch_rotate(const oscar::RotBatch& b, int d, cudaStream_t s) {
  const int path = g_rotate_path.load();
  RotKernel which[oscar::kRotMaxSegs];
  bool mixed = false;
  for (int i = 0; i < b.n; ++i) {
    which[i] = rotate_kernel_of<InT>(b.seg[i], d, sizeof(OutT), path);
    mixed = mixed || which[i] != which[0];
  }
  auto run = [&](const oscar::RotBatch& sub, RotKernel k) -> int {
    if (sub.n == 0) return OSCAR_OK;
    if (k == kRotTc) return launch_rotate_tc<InT, OutT>(sub, d, s);
    if (k == kRotBig)
      return d == 256 ? launch_rotate_big_d<InT, OutT, 256, 128>(sub, s)
                      : launch_rotate_big_d<InT, OutT, 128, 128>(sub, s);
    if (k == kRotMid)
      return d == 256 ? launch_rotate_big_d<InT, OutT, 256, 64>(sub, s) : launch_rotate_big_d<InT, OutT, 128, 64>(sub, s);
    return launch_rotate_fma<InT, OutT>(sub, d, s);
  };
  if (!mixed) return run(b, b.n > 0 ? which[0] : kRotSmall);
  for (RotKernel k : {kRotSmall, kRotMid, kRotBig, kRotTc}) {
    const int st = run(rotate_subset(b, [&](int i) { return which[i] == k; }), k);
    if (st) return st;
  }
  return OSCAR_OK;
}

// The kernel reads the rotation matrices before it waits for the launch in
// front of it, unless that launch may have written one: the outputs of this
// thread's previous rotation launch are remembered and checked for overlap.
// (No other library kernel writes anything a caller could pass as a rotation.)
void mark_rot_early(oscar::RotBatch& b, int out_dtype, int head_dim) {
  struct Range {
    uintptr_t lo, hi;
  };
  static thread_local Range prev[2 * oscar::kRotMaxSegs];
  static thread_local int n_prev = 0;
  const size_t out_es = out_dtype == OSCAR_DTYPE_F32 ? 4 : 2;
  const size_t rot_bytes = (size_t)head_dim * head_dim * sizeof(float);
  b.rot_early = 1;
  for (int i = 0; i < b.n; ++i) {
    const uintptr_t lo = reinterpret_cast<uintptr_t>(b.seg[i].rot), hi = lo + rot_bytes;
    for (int j = 0; j < n_prev; ++j)
      if (lo < prev[j].hi && prev[j].lo < hi) b.rot_early = 0;
  }
  n_prev = 0;
  for (int i = 0; i < b.n; ++i) {
    const oscar::RotSeg& d = b.seg[i];
    const int64_t last = (d.rows - 1) / d.heads;  // last token
    if (d.out != nullptr) {
      const uintptr_t lo = reinterpret_cast<uintptr_t>(d.out);
      prev[n_prev++] = {lo, lo + ((size_t)last * d.out_stride + (size_t)d.heads * head_dim) * out_es};
    }
    if (d.out_f32 != nullptr) {
      const uintptr_t lo = reinterpret_cast<uintptr_t>(d.out_f32);
      prev[n_prev++] = {lo, lo + ((size_t)last * d.out_f32_stride + (size_t)d.heads * head_dim) * 4};
    }
  }
}

template <typename InT>
int rotate_out(int out_dtype, const oscar::RotBatch& b, int d, cudaStream_t s) {
  if (out_dtype == OSCAR_DTYPE_F32) return launch_rotate<InT, float>(b, d, s);
  if (out_dtype == OSCAR_DTYPE_BF16) return launch_rotate<InT, __nv_bfloat16>(b, d, s);
  return launch_rotate<InT, __half>(b, d, s);
}

}  // namespace

extern "C" int oscar_rotate_rows_batch(const oscar_rotate_seg* segs, int32_t n_segs, int32_t x_dtype,
                                       int32_t head_dim, int32_t out_dtype, void* stream) {
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(OSCAR_ERR_INVALID, "rotate: D=%d must be 64, 128 or 256", head_dim);
  if (x_dtype < 0 || x_dtype > 2 || out_dtype < 0 || out_dtype > 2) return fail(OSCAR_ERR_INVALID, "rotate: bad dtype");
  if (n_segs < 0 || n_segs > oscar::kRotMaxSegs || (n_segs > 0 && segs == nullptr))
    return fail(OSCAR_ERR_INVALID, "rotate: 0 to %d segments", oscar::kRotMaxSegs);
  oscar::RotBatch b{};
  int64_t tiles = 0;
  for (int i = 0; i < n_segs; ++i) {
    const oscar_rotate_seg& g = segs[i];
    if (g.rows < 0) return fail(OSCAR_ERR_INVALID, "rotate: segment %d has %lld rows", i, (long long)g.rows);
    if (g.rows == 0 || (g.out == nullptr && g.out_f32 == nullptr)) continue;
    if (g.x == nullptr || g.rot == nullptr) return fail(OSCAR_ERR_INVALID, "rotate: null pointer in segment %d", i);
    if ((reinterpret_cast<uintptr_t>(g.rot) | reinterpret_cast<uintptr_t>(g.x)) & 15 || (g.rows > 1 && g.x_stride % 8))
      return fail(OSCAR_ERR_INVALID,
                  "rotate: x and the rotation must be 16-byte aligned, x rows a multiple of 8 elements apart");
    oscar::RotSeg& d = b.seg[b.n];
    d.x = g.x;
    d.rows = g.rows;
    d.x_stride = g.x_stride;
    d.rot = g.rot;
    d.transpose = g.transpose ? 1 : 0;
    d.out = g.out;
    d.out_stride = g.out_stride;
    d.out_f32 = g.out_f32;
    d.out_f32_stride = g.out_f32_stride;
    d.heads = 1;
    b.tile_begin[b.n] = (int)tiles;
    tiles += (g.rows + oscar::kRotRows - 1) / oscar::kRotRows;
    if (tiles > INT_MAX / 2) return fail(OSCAR_ERR_INVALID, "rotate: too many rows");
    ++b.n;
  }
  if (b.n == 0) return OSCAR_OK;
  b.tile_begin[b.n] = (int)tiles;
  mark_rot_early(b, out_dtype, head_dim);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (x_dtype == OSCAR_DTYPE_F32) return rotate_out<float>(out_dtype, b, head_dim, s);
  if (x_dtype == OSCAR_DTYPE_BF16) return rotate_out<__nv_bfloat16>(out_dtype, b, head_dim, s);
  return rotate_out<__half>(out_dtype, b, head_dim, s);
}

extern "C" int oscar_rotate_rows(const void* x, int32_t x_dtype, int64_t rows, int64_t x_stride, int32_t head_dim,
                                 const float* rot, int32_t transpose, void* out, int32_t out_dtype, int64_t out_stride,
                                 float* out_f32, int64_t out_f32_stride, void* stream) {
  oscar_rotate_seg g{x, rows, x_stride, rot, transpose, out, out_stride, out_f32, out_f32_stride};
  return oscar_rotate_rows_batch(&g, 1, x_dtype, head_dim, out == nullptr ? OSCAR_DTYPE_F32 : out_dtype, stream);
}

// ---------------------------------------------------------------------------
// One decode-sized layer step in one call (oscar_decode_layer_step).
namespace {

constexpr int64_t kStepAlign = 256;
inline int64_t step_align(int64_t x) { return (x + kStepAlign - 1) / kStepAlign * kStepAlign; }

struct StepScratch {
  int64_t k_rot, v_rot, k_lo, v_lo, q_lo, att, lse, ws;  // byte offsets
};

inline StepScratch step_scratch(int64_t n, int hq, int hk, int d, int es) {
  StepScratch s{};
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = off;
    off += step_align(bytes);
    return at;
  };
  s.k_rot = take(n * hk * d * 4);
  s.v_rot = take(n * hk * d * 4);
  s.k_lo = take(n * hk * d * es);
  s.v_lo = take(n * hk * d * es);
  s.q_lo = take(n * hq * d * es);
  s.att = take(n * hq * d * 4);
  s.lse = take(n * hq * 4);
  s.ws = off;
  return s;
}

template <typename T>
int step_rotations(const oscar::RotBatch& b, int out_dtype, int d, cudaStream_t s) {
  return rotate_out<T>(out_dtype, b, d, s);
}

}  // namespace

extern "C" int64_t oscar_decode_layer_step_scratch(int64_t n_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                                   int32_t head_dim, int32_t dtype) {
  if (n_tokens < 0 || num_q_heads < 1 || num_kv_heads < 1 || (dtype != OSCAR_DTYPE_BF16 && dtype != OSCAR_DTYPE_F16))
    return -1;
  return step_scratch(n_tokens, num_q_heads, num_kv_heads, head_dim, 2).ws;
}

extern "C" int oscar_decode_layer_step(
    const void* q, const void* k, const void* v, int32_t dtype, int64_t q_stride, int64_t k_stride, int64_t v_stride,
    int64_t n_tokens, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, const float* rot_k,
    const float* rot_v, const float* rot_vt, float k_clip_ratio, float v_clip_ratio, uint8_t* k_cache,
    uint8_t* v_cache, int64_t num_blocks, int32_t block_size, int64_t k_stride_block, int64_t k_stride_token,
    int64_t k_stride_head, int64_t v_stride_block, int64_t v_stride_token, int64_t v_stride_head,
    const int64_t* slot_mapping, const int32_t* qsl_dev, const int32_t* seqs_dev, const int32_t* block_table,
    int64_t bt_rows, int64_t bt_stride, const int32_t* qsl, const int32_t* seqs, int32_t num_requests,
    int32_t sink_eff, int32_t recent_tokens, float scale, float* stage_k, float* stage_v, int64_t* owner,
    int64_t stage_rows, void* out, int64_t out_stride, void* scratch, int64_t scratch_bytes, void* stream) {
  if (dtype != OSCAR_DTYPE_BF16 && dtype != OSCAR_DTYPE_F16)
    return fail(OSCAR_ERR_UNSUPPORTED, "layer step: query dtype must be bf16 or fp16");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(OSCAR_ERR_INVALID, "layer step: D=%d must be 64, 128 or 256", head_dim);
  if (n_tokens < 1 || num_q_heads < 1 || num_kv_heads < 1 || num_q_heads % num_kv_heads || !q || !k || !v || !out ||
      !scratch || !rot_k || !rot_v || !rot_vt || !qsl || !seqs)
    return fail(OSCAR_ERR_INVALID, "layer step: invalid arguments");
  if (q_stride < (int64_t)num_q_heads * head_dim || k_stride < (int64_t)num_kv_heads * head_dim ||
      v_stride < (int64_t)num_kv_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim ||
      (q_stride | k_stride | v_stride | out_stride) % 8)
    return fail(OSCAR_ERR_INVALID, "layer step: token strides must cover the heads and be multiples of 8 elements");
  if (num_requests < 1 || qsl[0] != 0 || qsl[num_requests] != n_tokens)
    return fail(OSCAR_ERR_INVALID, "Invalid slab query layout");
  for (int r = 0; r < num_requests; ++r)
    if (qsl[r + 1] - qsl[r] >= seqs[r] && qsl[r + 1] > qsl[r])
      return fail(OSCAR_ERR_UNSUPPORTED, "layer step: request %d has no cached history (prefix-free chunks take "
                  "the model-domain path)", r);
  const StepScratch sc = step_scratch(n_tokens, num_q_heads, num_kv_heads, head_dim, 2);
  if (scratch_bytes < sc.ws) return fail(OSCAR_ERR_INVALID, "layer step: scratch smaller than %lld bytes",
                                         (long long)sc.ws);
  if (reinterpret_cast<uintptr_t>(scratch) % kStepAlign)
    return fail(OSCAR_ERR_INVALID, "layer step: scratch must be %lld-byte aligned", (long long)kStepAlign);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  float* k_rot = reinterpret_cast<float*>(base + sc.k_rot);
  float* v_rot = reinterpret_cast<float*>(base + sc.v_rot);
  void* k_lo = base + sc.k_lo;
  void* v_lo = base + sc.v_lo;
  void* q_lo = base + sc.q_lo;
  float* att = reinterpret_cast<float*>(base + sc.att);
  float* lse = reinterpret_cast<float*>(base + sc.lse);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int hq = num_q_heads, hk = num_kv_heads, d = head_dim;
  // 1. k @ R_k, v @ R_v (fp32 for the store and the window, query dtype for the
  //    attention) and q @ R_k (query dtype), one launch
  {
    oscar::RotBatch b{};
    auto seg = [&](const void* x, int64_t stride, int heads, const float* rot, void* o, float* of) {
      oscar::RotSeg& g = b.seg[b.n];
      g.x = x;
      g.rows = n_tokens * heads;
      g.x_stride = stride;
      g.heads = heads;
      g.rot = rot;
      g.transpose = 0;
      g.out = o;
      g.out_stride = (int64_t)heads * d;
      g.out_f32 = of;
      g.out_f32_stride = (int64_t)heads * d;
      b.tile_begin[b.n] = b.n == 0 ? 0 : b.tile_begin[b.n - 1] + (int)((b.seg[b.n - 1].rows + oscar::kRotRows - 1) /
                                                                      oscar::kRotRows);
      ++b.n;
    };
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
         reinterpret_cast<uintptr_t>(rot_k) | reinterpret_cast<uintptr_t>(rot_v) |
         reinterpret_cast<uintptr_t>(rot_vt)) & 15)
      return fail(OSCAR_ERR_INVALID, "layer step: q / k / v and the rotations must be 16-byte aligned");
    seg(k, k_stride, hk, rot_k, k_lo, k_rot);
    seg(v, v_stride, hk, rot_v, v_lo, v_rot);
    seg(q, q_stride, hq, rot_k, q_lo, nullptr);
    b.tile_begin[b.n] = b.tile_begin[b.n - 1] + (int)((b.seg[b.n - 1].rows + oscar::kRotRows - 1) / oscar::kRotRows);
    mark_rot_early(b, dtype, d);
    const int st = dtype == OSCAR_DTYPE_BF16 ? step_rotations<__nv_bfloat16>(b, dtype, d, s)
                                             : step_rotations<__half>(b, dtype, d, s);
    if (st) return st;
  }
  // 2. clip + INT2 store and the staging write of the step's tokens
  int st = oscar_write_step(k_rot, v_rot, n_tokens, hk, d, k_clip_ratio, v_clip_ratio, k_cache, v_cache, num_blocks,
                            block_size, k_stride_block, k_stride_token, k_stride_head, v_stride_block,
                            v_stride_token, v_stride_head, slot_mapping, qsl_dev, seqs_dev, num_requests, sink_eff,
                            recent_tokens, stage_k, stage_v, owner, stage_rows, stream);
  if (st) return st;
  // 3. attention in the rotated space
  st = slab_attention_impl(q_lo, k_lo, v_lo, dtype, n_tokens, hq, hk, d, k_cache, v_cache, num_blocks, block_size,
                           k_stride_block, k_stride_token, k_stride_head, v_stride_block, v_stride_token,
                           v_stride_head, block_table, bt_rows, bt_stride, qsl, seqs, num_requests, scale, stage_k,
                           stage_v, owner, stage_rows, att, lse, base + sc.ws, scratch_bytes - sc.ws, stream, false);
  if (st) return st;
  // 4. o @ R_v^T into the output rows, in the query dtype
  {
    oscar::RotBatch b{};
    oscar::RotSeg& g = b.seg[0];
    g.x = att;
    g.rows = n_tokens * hq;
    g.x_stride = (int64_t)hq * d;
    g.heads = hq;
    g.rot = rot_vt;
    g.transpose = 0;
    g.out = out;
    g.out_stride = out_stride;
    g.out_f32 = nullptr;
    g.out_f32_stride = 0;
    b.n = 1;
    b.tile_begin[0] = 0;
    b.tile_begin[1] = (int)((g.rows + oscar::kRotRows - 1) / oscar::kRotRows);
    if (reinterpret_cast<uintptr_t>(out) & 15) return fail(OSCAR_ERR_INVALID, "layer step: out must be 16-byte aligned");
    mark_rot_early(b, dtype, d);
    st = rotate_out<float>(dtype, b, d, s);
  }
  return st;
}
