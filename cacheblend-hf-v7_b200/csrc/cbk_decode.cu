// Attention of one query token over the fused cache (a greedy decode step of
// the blended prefill: the reference's HF forward with past_key_values,
// runners.py:106-152).  out[hq] = softmax(scale q[hq] K[:p+1]^T) V[:p+1] per q
// head, keys 0..p of the cache rows, p read from device memory so that a
// captured decode step stays valid as the position advances.
//
// HBM-bound: every visible K/V byte is read once.  Grid (split, KV head); a CTA
// of eight warps takes a contiguous split of the keys (256, one 32-key pass per
// warp, while there are at most 64 splits) for the G q heads of its KV head.
// A pass: scores with one key per lane (the key row loaded in two halves; the G
// query rows, pre-scaled by scale * log2 e, sit in shared memory and are read
// as broadcasts), the first V rows issued, an online softmax per head across
// the warp, then P V with HD/32 head dimensions per lane and each key's weight
// broadcast by a shuffle (all 32 V rows issued before the softmax).  The warps
// merge through shared memory; the CTAs of a KV head merge without waiting:
// each stores its partial (running max, row sum, O) and counts, and the CTA
// that counts last merges them all (weights for every split staged in shared
// memory, then each output summed over the splits in increasing order, 16
// splits' loads in flight) and resets the counter.  fp32 throughout, output
// rounded once.
#include <algorithm>
#include <type_traits>

#include "cbk_common.cuh"

namespace cbk {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecMaxG = 8;
constexpr int kDecMaxSplits = 64;
constexpr int kDecSplit = kDecWarps * 32;   // keys per CTA pass: one 32-key pass per warp

struct DecLayout {
  int n_splits, split_len;
  size_t off_ml, off_o, off_cnt, bytes;
};

static size_t dec_align(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// splits of kDecSplit keys (one pass per warp) while they number <= kDecMaxSplits,
// longer splits (several passes per warp) beyond
static DecLayout dec_layout(int64_t cap, int n_kv_heads, int G, int head_dim) {
  DecLayout d;
  const int64_t want = (cap + kDecSplit - 1) / kDecSplit;
  d.n_splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, kDecMaxSplits)));
  const int64_t per = (cap + d.n_splits - 1) / d.n_splits;
  d.split_len = static_cast<int>((per + kDecSplit - 1) / kDecSplit * kDecSplit);
  const size_t parts = static_cast<size_t>(n_kv_heads) * d.n_splits * G;
  d.off_ml = 0;
  d.off_o = dec_align(parts * sizeof(float2));
  d.off_cnt = d.off_o + dec_align(parts * head_dim * sizeof(float));
  d.bytes = d.off_cnt + dec_align(static_cast<size_t>(n_kv_heads) * sizeof(int));
  return d;
}

template <int DT, int HD, int G>
__global__ void __launch_bounds__(kDecThreads, 2)
decode_attn_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                   const uint16_t* __restrict__ vc, int64_t kv_stride, const int64_t* __restrict__ pos,
                   int64_t cap, float scale_log2, int split_len, float2* part_ml, float* part_o, int* cnt,
                   uint16_t* __restrict__ out, int32_t* status) {
  using E = Elem<DT>;
  constexpr int kDimLane = HD / 32;                  // head dimensions per lane in P V
  constexpr int kKPart = 4;                          // 16-byte vectors of the key row per load batch
  constexpr int kKParts = HD / 8 / kKPart;
  using VRaw = typename std::conditional<kDimLane == 4, uint2, uint32_t>::type;
  __shared__ __align__(16) float s_q[G][HD];
  __shared__ float s_m[kDecWarps][G], s_l[kDecWarps][G];
  __shared__ __align__(16) float s_o[kDecWarps][G][HD];
  __shared__ float2 s_ml[kDecMaxSplits][G];
  __shared__ float s_w[kDecMaxSplits][G];
  __shared__ float s_L[G];
  __shared__ int s_last;
  const int h = blockIdx.y, split = blockIdx.x, n_splits = gridDim.x;
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
  const uint16_t* vh = vc + static_cast<int64_t>(h) * HD + lane * kDimLane;
  for (int64_t c = k0 + warp * 32; c < k1; c += kDecWarps * 32) {
    // scores, one key per lane, the key row in parts of kKPart vectors
    const int64_t key = c + lane;
    const bool valid = key < k1;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (valid) {
      const uint16_t* kr = kh + key * kv_stride;
#pragma unroll
      for (int part = 0; part < kKParts; ++part) {
        uint4 kv4[kKPart];
#pragma unroll
        for (int v = 0; v < kKPart; ++v) kv4[v] = ld_vec(kr + (part * kKPart + v) * 8);
#pragma unroll
        for (int v = 0; v < kKPart; ++v) {
          const int e0 = (part * kKPart + v) * 8;
          const uint16_t* hk = reinterpret_cast<const uint16_t*>(&kv4[v]);
          float kf[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) kf[e] = E::to_f(hk[e]);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float4 qa = *reinterpret_cast<const float4*>(&s_q[g][e0]);
            const float4 qb = *reinterpret_cast<const float4*>(&s_q[g][e0 + 4]);
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
    }
    const int nk = static_cast<int>(std::min<int64_t>(32, k1 - c));
    constexpr int kVBatch = 8;
    VRaw raw[kVBatch];
#pragma unroll
    for (int jj = 0; jj < kVBatch; ++jj)
      if (jj < nk) raw[jj] = *reinterpret_cast<const VRaw*>(vh + (c + jj) * kv_stride);
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
#pragma unroll
    for (int j0 = 0; j0 < 32; j0 += kVBatch) {
      if (j0 >= nk) break;
      VRaw cur[kVBatch];
#pragma unroll
      for (int jj = 0; jj < kVBatch; ++jj) cur[jj] = raw[jj];
      if (j0 + kVBatch < 32) {
#pragma unroll
        for (int jj = 0; jj < kVBatch; ++jj)
          if (j0 + kVBatch + jj < nk)
            raw[jj] = *reinterpret_cast<const VRaw*>(vh + (c + j0 + kVBatch + jj) * kv_stride);
      }
#pragma unroll
      for (int jj = 0; jj < kVBatch; ++jj) {
        if (j0 + jj >= nk) break;
        const uint16_t* hv = reinterpret_cast<const uint16_t*>(&cur[jj]);
        float vf[kDimLane];
#pragma unroll
        for (int d = 0; d < kDimLane; ++d) vf[d] = E::to_f(hv[d]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pj = __shfl_sync(0xffffffffu, pw[g], j0 + jj);
#pragma unroll
          for (int d = 0; d < kDimLane; ++d) o[g][d] = fmaf(pj, vf[d], o[g][d]);
        }
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
    const int64_t part = (static_cast<int64_t>(h) * n_splits + split) * G + g;
    part_o[part * HD + d] = acc;                     // O un-normalised, relative to M
    if (d == 0) part_ml[part] = make_float2(M, L);
  }
  // the CTA that counts last for this KV head merges every split
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&cnt[h], 1) == n_splits - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) cnt[h] = 0;                          // ready for the next call
  const int64_t base = static_cast<int64_t>(h) * n_splits * G;
  for (int i = tid; i < n_splits * G; i += kDecThreads) s_ml[i / G][i % G] = __ldcg(&part_ml[base + i]);
  __syncthreads();
  if (tid < G) {
    const int g = tid;
    float M = -INFINITY;
    for (int sp = 0; sp < n_splits; ++sp)
      if (s_ml[sp][g].y > 0.f) M = fmaxf(M, s_ml[sp][g].x);
    float L = 0.f;
    for (int sp = 0; sp < n_splits; ++sp) {
      const float wt = s_ml[sp][g].y > 0.f ? ex2(s_ml[sp][g].x - M) : 0.f;
      s_w[sp][g] = wt;
      L += wt * s_ml[sp][g].y;
    }
    s_L[g] = L;
  }
  __syncthreads();
  // each output summed over the splits, kSpBatch splits' loads in flight
  constexpr int kSpBatch = 16;
#pragma unroll 1
  for (int i = tid; i < G * HD; i += kDecThreads) {
    const int g = i / HD, d = i % HD;
    const float* po = part_o + (base + g) * HD + d;  // split sp at po[sp * G * HD]
    float acc = 0.f;
    for (int sp0 = 0; sp0 < n_splits; sp0 += kSpBatch) {
      float x[kSpBatch];
#pragma unroll
      for (int u = 0; u < kSpBatch; ++u)
        x[u] = sp0 + u < n_splits ? __ldcg(po + static_cast<int64_t>(sp0 + u) * G * HD) : 0.f;
#pragma unroll
      for (int u = 0; u < kSpBatch; ++u)
        if (sp0 + u < n_splits) acc = fmaf(s_w[sp0 + u][g], x[u], acc);
    }
    out[(static_cast<int64_t>(h) * G + g) * HD + d] = E::from_f(acc / s_L[g]);
  }
}

}  // namespace cbk

using namespace cbk;

extern "C" size_t cbk_decode_attn_workspace_bytes(int64_t cap, int n_q_heads, int n_kv_heads, int head_dim) {
  if (cap <= 0 || n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads != 0) return 0;
  return dec_layout(cap, n_kv_heads, n_q_heads / n_kv_heads, head_dim).bytes;
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
  const DecLayout lay = dec_layout(cap, n_kv_heads, G, head_dim);
  if (workspace_bytes < lay.bytes)
    return set_error(CBK_ERR_WORKSPACE, "cbk_decode_attn: workspace %zu < %zu bytes", workspace_bytes, lay.bytes);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto ml = reinterpret_cast<float2*>(ws + lay.off_ml);
  auto po = reinterpret_cast<float*>(ws + lay.off_o);
  auto cnt = reinterpret_cast<int*>(ws + lay.off_cnt);
  const dim3 grid(lay.n_splits, n_kv_heads);
  auto st = static_cast<cudaStream_t>(stream);
  const float sl2 = scale * 1.4426950408889634f;
  auto qp = static_cast<const uint16_t*>(q);
  auto kp = static_cast<const uint16_t*>(k_cache);
  auto vp = static_cast<const uint16_t*>(v_cache);
  auto op = static_cast<uint16_t*>(out);
#define CBK_DEC3(DT, HD, GG)                                                                            \
  decode_attn_kernel<DT, HD, GG><<<grid, kDecThreads, 0, st>>>(qp, kp, vp, kv_row_stride, pos, cap, sl2,   \
                                                              lay.split_len, ml, po, cnt, op, status)
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
