// Attention of one query token over the fused cache (a greedy decode step of
// the blended prefill: the reference's HF forward with past_key_values,
// runners.py:106-152).  out[hq] = softmax(scale q[hq] K[:p+1]^T) V[:p+1] per q
// head, keys 0..p of the cache rows, p read from device memory so that a
// captured decode step stays valid as the position advances.
//
// HBM-bound: every visible K/V byte is read once.  Grid (split, KV head),
// about two CTAs per SM; a CTA of four warps takes a contiguous split of the
// keys for the G q heads of its KV head, each warp 32 keys per pass.  A pass
// copies its 32 K rows and 32 V rows into shared memory with cp.async, 16
// lanes per row and every copy in flight at once; scores are computed one key
// per lane (K rows padded by 16 bytes so these reads do not conflict; the G
// query rows, pre-scaled by scale * log2 e, are read as broadcasts), then an
// online softmax per head across the warp and P V with HD/32 head dimensions
// per lane, each key's weight broadcast by a shuffle.  The warps merge through
// shared memory into the split's partial (running max, row sum, O), and a
// second small kernel merges the splits (one CTA per q head, one thread per
// head dimension, every split's load in flight): a merge inside the first
// kernel by its last CTA measured slower (22.3 us against 17.9 us for the two
// kernels at 32 q / 8 KV heads and 6209 keys), as a handful of CTAs then
// finished the launch alone.  fp32 throughout, output
// rounded once.
#include <algorithm>
#include <type_traits>

#include "cbk_common.cuh"

namespace cbk {

int sm_count_layer();   // cbk_layer.cu
int ensure_smem_attr(const void* func, int bytes);   // cbk_api.cu

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecMaxSplits = 64;
constexpr int kDecPass = 32;                 // keys per warp pass
constexpr int kDecCtaKeys = kDecWarps * kDecPass;

struct DecLayout {
  int n_splits, split_len;
  size_t off_ml, off_o, bytes;
};

static size_t dec_align(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace sized for kDecMaxSplits splits (independent of the device); the
// split count fills one wave of two CTAs per SM: about 2 * SMs / n_kv_heads
// splits (fewer when the cache is short), each a multiple of 32 keys.
static DecLayout dec_layout(int64_t cap, int n_kv_heads, int G, int head_dim, int sms) {
  DecLayout d;
  const int64_t by_keys = (cap + kDecCtaKeys - 1) / kDecCtaKeys;
  const int64_t by_sms = std::max<int64_t>(1, 2LL * sms / n_kv_heads);
  d.n_splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({by_keys, by_sms, kDecMaxSplits})));
  const int64_t per = (cap + d.n_splits - 1) / d.n_splits;
  d.split_len = static_cast<int>((per + kDecPass - 1) / kDecPass * kDecPass);
  const size_t parts = static_cast<size_t>(n_kv_heads) * kDecMaxSplits * G;
  d.off_ml = 0;
  d.off_o = dec_align(parts * sizeof(float2));
  d.bytes = d.off_o + dec_align(parts * head_dim * sizeof(float));
  return d;
}

// dynamic shared memory: per warp a K tile (32 rows, pitch HD + 8 elements so
// that one key per lane reads without bank conflicts) and a V tile (32 rows)
template <int HD>
struct DecSmem {
  static constexpr int kKPitch = HD + 8;
  static constexpr int kKTile = kDecPass * kKPitch;     // elements
  static constexpr int kVTile = kDecPass * HD;
  static constexpr int kBytes = kDecWarps * (kKTile + kVTile) * 2;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

template <int DT, int HD, int G>
__global__ void __launch_bounds__(kDecThreads, 2)
decode_attn_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                   const uint16_t* __restrict__ vc, int64_t kv_stride, const int64_t* __restrict__ pos,
                   int64_t cap, float scale_log2, int split_len, float2* part_ml, float* part_o,
                   int32_t* status) {
  using E = Elem<DT>;
  using SM = DecSmem<HD>;
  constexpr int kDimLane = HD / 32;                  // head dimensions per lane in P V
  constexpr int kVecRow = HD / 8;                    // 16-byte pieces of a row
  using VRaw = typename std::conditional<kDimLane == 4, uint2, uint32_t>::type;
  extern __shared__ __align__(16) uint16_t s_kv[];
  __shared__ __align__(16) float s_q[G][HD];
  __shared__ float s_m[kDecWarps][G], s_l[kDecWarps][G];
  __shared__ __align__(16) float s_o[kDecWarps][G][HD];
  const int h = blockIdx.y, split = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t p = *pos;
  if (p < 0 || p >= cap) {                           // nothing visible: reported, output left alone
    if (tid == 0 && split == 0) report(status, CBK_STATUS_BAD_INDEX);
    return;
  }
  const int64_t n_keys = p + 1;
  for (int i = tid; i < G * HD; i += kDecThreads)
    s_q[i / HD][i % HD] = E::to_f(q[(static_cast<int64_t>(h) * G + i / HD) * HD + i % HD]) * scale_log2;
  __syncthreads();

  uint16_t* sk = s_kv + warp * SM::kKTile;
  uint16_t* sv = s_kv + kDecWarps * SM::kKTile + warp * SM::kVTile;
  float m[G], l[G], o[G][kDimLane];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < kDimLane; ++d) o[g][d] = 0.f;
  }
  const int64_t k0 = static_cast<int64_t>(split) * split_len;
  const int64_t k1 = std::min<int64_t>(k0 + split_len, n_keys);
  const uint16_t* kh = kc + static_cast<int64_t>(h) * HD;
  const uint16_t* vh = vc + static_cast<int64_t>(h) * HD;
  for (int64_t c = k0 + warp * kDecPass; c < k1; c += kDecWarps * kDecPass) {
    const int nk = static_cast<int>(std::min<int64_t>(kDecPass, k1 - c));
    // the pass's K and V rows into shared memory, every copy in flight at once
    // (16 lanes per row: coalesced)
    __syncwarp();                                    // the previous pass is done with the tiles
#pragma unroll
    for (int i = 0; i < kDecPass * kVecRow / 32; ++i) {
      const int idx = lane + 32 * i;
      const int r = idx / kVecRow, v = idx % kVecRow;
      if (r < nk) {
        cp_async16(sk + r * SM::kKPitch + v * 8, kh + (c + r) * kv_stride + v * 8);
        cp_async16(sv + r * HD + v * 8, vh + (c + r) * kv_stride + v * 8);
      }
    }
    cp_async_wait_all();
    __syncwarp();
    // scores, one key per lane
    const bool valid = lane < nk;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (valid) {
      const uint16_t* kr = sk + lane * SM::kKPitch;
#pragma unroll 4
      for (int v = 0; v < kVecRow; ++v) {
        const uint4 kv4 = *reinterpret_cast<const uint4*>(kr + v * 8);
        const uint16_t* hk = reinterpret_cast<const uint16_t*>(&kv4);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) kf[e] = E::to_f(hk[e]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 qa = *reinterpret_cast<const float4*>(&s_q[g][v * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&s_q[g][v * 8 + 4]);
          s[g] = fmaf(qa.x, kf[0], s[g]);
          s[g] = fmaf(qa.y, kf[1], s[g]);
          s[g] = fmaf(qa.z, kf[2], s[g]);
          s[g] = fmaf(qa.w, kf[3], s[g]);
          s[g] = fmaf(qb.x, kf[4], s[g]);
          s[g] = fmaf(qb.y, kf[5], s[g]);
          s[g] = fmaf(qb.z, kf[6], s[g]);
          s[g] = fmaf(qb.w, kf[7], s[g]);
        }
      }
    }
    // online softmax per head (lane 0's key is valid, so every max is finite)
    float pw[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = valid ? s[g] : -INFINITY;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m[g], mx);
      const float alpha = ex2(m[g] - m_new);
      pw[g] = valid ? ex2(s[g] - m_new) : 0.f;
      float sum = pw[g];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l[g] = l[g] * alpha + sum;
      m[g] = m_new;
#pragma unroll
      for (int d = 0; d < kDimLane; ++d) o[g][d] *= alpha;
    }
    // P V, keys in order, kDimLane dimensions per lane from the V tile
#pragma unroll 8
    for (int j = 0; j < nk; ++j) {
      const VRaw raw = *reinterpret_cast<const VRaw*>(sv + j * HD + lane * kDimLane);
      const uint16_t* hv = reinterpret_cast<const uint16_t*>(&raw);
      float vf[kDimLane];
#pragma unroll
      for (int d = 0; d < kDimLane; ++d) vf[d] = E::to_f(hv[d]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = __shfl_sync(0xffffffffu, pw[g], j);
#pragma unroll
        for (int d = 0; d < kDimLane; ++d) o[g][d] = fmaf(pj, vf[d], o[g][d]);
      }
    }
  }
  // merge the warps (a warp without keys has l = 0)
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
#pragma unroll
    for (int d = 0; d < kDimLane; ++d) s_o[warp][g][lane * kDimLane + d] = o[g][d];
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += kDecThreads) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w)
      if (s_l[w][g] > 0.f) M = fmaxf(M, s_m[w][g]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float wt = s_l[w][g] > 0.f ? ex2(s_m[w][g] - M) : 0.f;
      L += wt * s_l[w][g];
      acc += wt * s_o[w][g][d];
    }
    const int64_t part = (static_cast<int64_t>(h) * kDecMaxSplits + split) * G + g;
    part_o[part * HD + d] = acc;                     // O un-normalised, relative to M
    if (d == 0) part_ml[part] = make_float2(M, L);
  }
}

// Merge of the splits, one CTA per (KV head, q head of its group), one thread
// per head dimension: O = sum_s w_s O_s / sum_s w_s l_s, w_s = 2^(m_s - M)
// over splits with visible keys, every split's load in flight at once, sums
// in increasing split order.
template <int DT, int HD>
__global__ void __launch_bounds__(HD)
decode_merge_kernel(const float2* __restrict__ part_ml, const float* __restrict__ part_o, int G, int n_splits,
                    const int64_t* __restrict__ pos, int64_t cap, uint16_t* __restrict__ out) {
  using E = Elem<DT>;
  __shared__ float s_w[kDecMaxSplits], s_l[kDecMaxSplits];
  __shared__ float s_M, s_L;
  const int h = blockIdx.x / G, g = blockIdx.x % G, d = threadIdx.x;
  const int64_t p = *pos;
  if (p < 0 || p >= cap) return;                     // reported by the attention kernel
  const int64_t base = (static_cast<int64_t>(h) * kDecMaxSplits) * G + g;   // split s at base + s * G
  float x[kDecMaxSplits];
#pragma unroll
  for (int sp = 0; sp < kDecMaxSplits; ++sp)
    x[sp] = sp < n_splits ? part_o[(base + static_cast<int64_t>(sp) * G) * HD + d] : 0.f;
  if (d < n_splits) {
    const float2 ml = part_ml[base + static_cast<int64_t>(d) * G];
    s_w[d] = ml.x;
    s_l[d] = ml.y;
  }
  __syncthreads();
  if (d == 0) {
    float M = -INFINITY;
    for (int sp = 0; sp < n_splits; ++sp)
      if (s_l[sp] > 0.f) M = fmaxf(M, s_w[sp]);
    s_M = M;
  }
  __syncthreads();
  if (d < n_splits) s_w[d] = s_l[d] > 0.f ? ex2(s_w[d] - s_M) : 0.f;
  __syncthreads();
  if (d == 0) {
    float L = 0.f;
    for (int sp = 0; sp < n_splits; ++sp) L += s_w[sp] * s_l[sp];
    s_L = L;
  }
  __syncthreads();
  float acc = 0.f;
#pragma unroll
  for (int sp = 0; sp < kDecMaxSplits; ++sp)
    if (sp < n_splits) acc = fmaf(s_w[sp], x[sp], acc);
  out[(static_cast<int64_t>(h) * G + g) * HD + d] = E::from_f(acc / s_L);
}

}  // namespace cbk

using namespace cbk;

extern "C" size_t cbk_decode_attn_workspace_bytes(int64_t cap, int n_q_heads, int n_kv_heads, int head_dim) {
  if (cap <= 0 || n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads != 0) return 0;
  return dec_layout(cap, n_kv_heads, n_q_heads / n_kv_heads, head_dim, sm_count_layer()).bytes;
}

extern "C" int cbk_decode_attn(const void* q, const void* k_cache, const void* v_cache, int64_t kv_row_stride,
                               const int64_t* pos, int64_t cap, int n_q_heads, int n_kv_heads, int head_dim,
                               float scale, int dtype, void* out, void* workspace, size_t workspace_bytes,
                               int32_t* status, void* stream) {
  if (dtype != CBK_BF16 && dtype != CBK_F16)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_decode_attn: dtype %d not supported", dtype);
  if (head_dim != 64 && head_dim != 128)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_decode_attn: head_dim %d (64 or 128 only)", head_dim);
  if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads != 0)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_decode_attn: n_q_heads must be a multiple of n_kv_heads");
  {
    const int g = n_q_heads / n_kv_heads;
    if (g != 1 && g != 2 && g != 4 && g != 8)
      return set_error(CBK_ERR_UNSUPPORTED, "cbk_decode_attn: q heads per KV head %d not in {1, 2, 4, 8}", g);
  }
  if (cap <= 0 || kv_row_stride < static_cast<int64_t>(n_kv_heads) * head_dim || kv_row_stride % 8 != 0)
    return set_error(CBK_ERR_INVALID, "cbk_decode_attn: bad cache rows (cap %lld, stride %lld)", (long long)cap,
                     (long long)kv_row_stride);
  if (!q || !k_cache || !v_cache || !pos || !out || !workspace)
    return set_error(CBK_ERR_INVALID, "cbk_decode_attn: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(workspace)) & 15u)
    return set_error(CBK_ERR_INVALID, "cbk_decode_attn: caches and workspace must be 16-byte aligned");
  const int G = n_q_heads / n_kv_heads;
  const DecLayout lay = dec_layout(cap, n_kv_heads, G, head_dim, sm_count_layer());
  if (workspace_bytes < lay.bytes)
    return set_error(CBK_ERR_WORKSPACE, "cbk_decode_attn: workspace %zu < %zu bytes", workspace_bytes, lay.bytes);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto ml = reinterpret_cast<float2*>(ws + lay.off_ml);
  auto po = reinterpret_cast<float*>(ws + lay.off_o);
  const dim3 grid(lay.n_splits, n_kv_heads);
  auto st = static_cast<cudaStream_t>(stream);
  const float sl2 = scale * 1.4426950408889634f;
  auto qp = static_cast<const uint16_t*>(q);
  auto kp = static_cast<const uint16_t*>(k_cache);
  auto vp = static_cast<const uint16_t*>(v_cache);
  auto op = static_cast<uint16_t*>(out);
#define CBK_DEC3(DT, HD, GG)                                                                            \
  do {                                                                                                  \
    auto kern = decode_attn_kernel<DT, HD, GG>;                                                         \
    if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), DecSmem<HD>::kBytes)) return rc; \
    kern<<<grid, kDecThreads, DecSmem<HD>::kBytes, st>>>(qp, kp, vp, kv_row_stride, pos, cap, sl2,       \
                                                        lay.split_len, ml, po, status);                 \
    decode_merge_kernel<DT, HD><<<n_kv_heads * GG, HD, 0, st>>>(ml, po, GG, lay.n_splits, pos, cap, op);  \
  } while (0)
#define CBK_DEC(DT, HD)                                                                                 \
  switch (G) {                                                                                          \
    case 1: CBK_DEC3(DT, HD, 1); break;                                                                 \
    case 2: CBK_DEC3(DT, HD, 2); break;                                                                 \
    case 4: CBK_DEC3(DT, HD, 4); break;                                                                 \
    default: CBK_DEC3(DT, HD, 8); break;                                                                \
  }
  if (dtype == CBK_BF16) {
    if (head_dim == 128) { CBK_DEC(CBK_BF16, 128); } else { CBK_DEC(CBK_BF16, 64); }
  } else {
    if (head_dim == 128) { CBK_DEC(CBK_F16, 128); } else { CBK_DEC(CBK_F16, 64); }
  }
#undef CBK_DEC
#undef CBK_DEC3
  return check_launch("decode_attn_kernel");
}
