// HKVD: per-token K deviation and top-K selection with the force-include rule.
//
// Deviation order (reproduced bit-for-bit by the oracle):
//   the row's features are cut into 16-byte vectors of 8 elements; each
//   vector's sum of squared differences is taken in element order,
//   s = d_0*d_0, s = s + d_e*d_e (separately rounded fp32 ops, no FMA,
//   d_e = new - old); the row total is the complete binary tree of pairwise
//   fp32 adds over the vector sums, padded with zeros to a power of two
//   (node = left + right, adjacent nodes paired level by level).
//   Any aligned power-of-two run of vectors is a subtree, so the deviation of
//   a slice of heads (one rank's KV heads when the heads are sharded over
//   ranks) is a node of the full tree, and combining the slices' values with
//   the same pairwise tree reproduces the single-GPU bits.
//   In the kernel: one warp per token; lane l holds vectors l, l+32, l+64,
//   l+96 of each 128-vector group; an xor butterfly over the lanes (1, 2, 4, 8,
//   16) forms the 32-vector nodes, two more adds the 128-vector node, and
//   successive groups are merged by a binary counter (which equals the
//   zero-padded complete tree).
//
// Top-K: one CTA.  Order keys are the fp32 bit patterns mapped to a monotone
// unsigned order; four 8-bit radix passes find the k-th largest key T and how
// many elements equal to T are taken (lowest index first).  An order-preserving
// compaction then writes the ascending index list.  Up to 33792 keys, each
// thread holds a run of consecutive keys in registers and the compaction is one
// block-wide scan; above that, keys are cached in shared memory (up to 40960) or
// re-read, each warp walks a chunk, and the compaction is per warp.  In
// hkvd_select the top-K kernel is a programmatic dependent of the deviation
// kernel, so its launch overlaps the deviation's tail.
#include <mutex>

#include "cbk_common.cuh"

namespace cbk {

constexpr int kDevThreads = 256;
constexpr int kDevBatch = 4;     // 16-byte vectors per lane per batch
constexpr int kDevLevels = 16;   // counter levels: rows of up to 2^16 groups of 128 vectors
constexpr int64_t kDevMaxFeat = (int64_t{1} << kDevLevels) * 32 * kDevBatch * 8;

template <int DT>
__device__ __forceinline__ float vec_sq_sum(const uint4& x, const uint4& y) {
  const uint16_t* xs = reinterpret_cast<const uint16_t*>(&x);
  const uint16_t* ys = reinterpret_cast<const uint16_t*>(&y);
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float d = __fsub_rn(Elem<DT>::to_f(xs[e]), Elem<DT>::to_f(ys[e]));
    s = e ? __fadd_rn(s, __fmul_rn(d, d)) : __fmul_rn(d, d);
  }
  return s;
}

template <int DT>
__global__ void __launch_bounds__(kDevThreads)
deviation_kernel(const uint16_t* __restrict__ k_new, int64_t new_stride,
                 const cbk_chunk_src* __restrict__ old_srcs, const int64_t* __restrict__ chunk_start,
                 int n_chunks, int64_t S, int64_t feat, float* __restrict__ dev) {
  const int lane = threadIdx.x & 31;
  // the top-K kernel that follows in hkvd_select is a programmatic dependent: it may
  // be placed once every CTA of this grid has started, and waits for this grid's end
  asm volatile("griddepcontrol.launch_dependents;");
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * kDevThreads + threadIdx.x) >> 5;
  if (t >= S) return;
  // A lane's vectors of a 128-vector group are loaded together (the fresh
  // row's first group before the chunk search), then summed.
  const uint16_t* a = k_new + t * new_stride;
  const int nvec = static_cast<int>(feat >> 3);
  uint4 x[kDevBatch], y[kDevBatch];
#pragma unroll
  for (int q = 0; q < kDevBatch; ++q)
    if (lane + q * 32 < nvec) x[q] = ld_vec(a + (lane + q * 32) * 8);
  int lo = 0, hi = n_chunks - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (chunk_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const uint16_t* b = static_cast<const uint16_t*>(old_srcs[lo].k) + (t - chunk_start[lo]) * feat;
  // binary counter over 128-vector group nodes: stack[i] holds a node of 2^i
  // groups (constant indices after unrolling, so the stack stays in registers)
  float stack[kDevLevels];
  int groups = 0;
  for (int v0 = 0; v0 < nvec; v0 += 32 * kDevBatch) {
    if (v0) {
#pragma unroll
      for (int q = 0; q < kDevBatch; ++q)
        if (v0 + lane + q * 32 < nvec) x[q] = ld_vec(a + (v0 + lane + q * 32) * 8);
    }
#pragma unroll
    for (int q = 0; q < kDevBatch; ++q)
      if (v0 + lane + q * 32 < nvec) y[q] = ld_stream(b + (v0 + lane + q * 32) * 8);
    float n32[kDevBatch];
#pragma unroll
    for (int q = 0; q < kDevBatch; ++q) {
      float s = (v0 + lane + q * 32 < nvec) ? vec_sq_sum<DT>(x[q], y[q]) : 0.f;
#pragma unroll
      for (int o = 1; o <= 16; o <<= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      n32[q] = s;                                           // vectors [v0 + 32q, +32)
    }
    float node = __fadd_rn(__fadd_rn(n32[0], n32[1]), __fadd_rn(n32[2], n32[3]));   // 128 vectors
#pragma unroll
    for (int lvl = 0; lvl < kDevLevels; ++lvl) {
      if (!((groups >> lvl) & 1)) {
        stack[lvl] = node;
        break;
      }
      node = __fadd_rn(stack[lvl], node);
    }
    ++groups;
  }
  // fold what the counter holds, from the smallest node up (the zero padding
  // of the complete tree leaves the smaller node as the right operand)
  float acc = 0.f;
  bool have = false;
#pragma unroll
  for (int lvl = 0; lvl < kDevLevels; ++lvl) {
    if ((groups >> lvl) & 1) {
      acc = have ? __fadd_rn(stack[lvl], acc) : stack[lvl];
      have = true;
    }
  }
  if (lane == 0) dev[t] = acc;
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int64_t kTopkSmemKeys = 40960;   // keys cached in shared memory up to this S
constexpr int kTopkUnroll = 8;             // 32-key tiles whose loads are issued together

// Each warp owns one contiguous chunk of the keys (a multiple of 32 long) and
// walks it in 32-key tiles, lane = key within the tile: loads are coalesced,
// shared-memory reads conflict-free, and within a warp the keys come in index
// order, which the ordered compaction below relies on.
__global__ void __launch_bounds__(kTopkThreads, 1)
topk_kernel(const float* __restrict__ dev, int64_t S, int64_t k, int force_last,
            int64_t* __restrict__ idx, int32_t* status) {
  extern __shared__ uint32_t s_keys[];   // S keys when S <= kTopkSmemKeys
  __shared__ uint32_t s_hist[256];
  __shared__ uint32_t s_wa[kTopkWarps], s_wb[kTopkWarps];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int64_t s_krem, s_total_eq;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // launched as a programmatic dependent of the deviation kernel (a no-op otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bool cached = S <= kTopkSmemKeys;
  const int64_t chunk = ((S + kTopkWarps - 1) / kTopkWarps + 31) & ~int64_t{31};
  const int64_t w_lo = warp * chunk, w_hi = w_lo + chunk < S ? w_lo + chunk : S;
  if (cached)
    for (int64_t i = tid; i < S; i += kTopkThreads) s_keys[i] = order_key(dev[i]);
  for (int b = tid; b < 256; b += kTopkThreads) s_hist[b] = 0;
  if (tid == 0) { s_prefix = 0; s_mask = 0; s_krem = k; }
  __syncthreads();
  auto key_at = [&](int64_t i) { return cached ? s_keys[i] : order_key(dev[i]); };

  // four 8-bit radix passes, high digit first (shared-memory atomics; lanes
  // that hit one bin are serialised by the hardware, a few cycles per warp)
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int64_t b = w_lo; b < w_hi; b += 32 * kTopkUnroll) {
      uint32_t key[kTopkUnroll];            // all loads of the batch first (L2 round trips overlap)
#pragma unroll
      for (int u = 0; u < kTopkUnroll; ++u) {
        const int64_t i = b + u * 32 + lane;
        key[u] = i < w_hi ? key_at(i) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kTopkUnroll; ++u) {
        const int64_t i = b + u * 32 + lane;
        if (i < w_hi && (key[u] & mask) == prefix) atomicAdd(&s_hist[(key[u] >> shift) & 255u], 1u);
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l sums the 8 digits 255-8l .. 248-8l (descending digit order)
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) { c[e] = s_hist[255 - 8 * lane - e]; sum += c[e]; }
#pragma unroll
      for (int e = 0; e < 8; ++e) s_hist[255 - 8 * lane - e] = 0;      // ready for the next pass
      uint32_t incl = sum;   // inclusive scan over lanes: counts of digits >= this lane's lowest
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const uint32_t excl = incl - sum;
      const int64_t krem = s_krem;
      const bool here = (excl < krem) && (incl >= krem);
      const unsigned who = __ballot_sync(0xffffffffu, here);
      if (here && lane == __ffs(who) - 1) {
        uint32_t above = excl;
        for (int e = 0; e < 8; ++e) {
          if (above + c[e] >= krem) {
            const uint32_t digit = 255 - 8 * lane - e;
            s_prefix = prefix | (digit << shift);
            s_mask = mask | (255u << shift);
            s_krem = krem - above;
            s_total_eq = c[e];
            break;
          }
          above += c[e];
        }
      }
    }
    __syncthreads();
  }

  const uint32_t T = s_prefix;
  const int64_t k_eq = s_krem;          // elements equal to T that are taken (lowest index first)
  const int64_t total_eq = s_total_eq;  // elements equal to T in total
  const uint32_t last_key = key_at(S - 1);
  const bool last_sel = last_key > T || (last_key == T && total_eq <= k_eq);
  const bool force = force_last && !last_sel;

  // ordered compaction: per-warp counts, warp offsets, then each warp writes its keys
  const unsigned lt_mask = (1u << lane) - 1u;
  uint32_t n_gt = 0, n_eq = 0;
  for (int64_t b = w_lo; b < w_hi; b += 32 * kTopkUnroll) {
    uint32_t key[kTopkUnroll];
#pragma unroll
    for (int u = 0; u < kTopkUnroll; ++u) {
      const int64_t i = b + u * 32 + lane;
      key[u] = i < w_hi ? key_at(i) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kTopkUnroll; ++u) {
      const bool in = b + u * 32 + lane < w_hi;
      n_gt += __popc(__ballot_sync(0xffffffffu, in && key[u] > T));
      n_eq += __popc(__ballot_sync(0xffffffffu, in && key[u] == T));
    }
  }
  if (lane == 0) {
    s_wa[warp] = n_gt;
    s_wb[warp] = n_eq;
  }
  __syncthreads();
  if (warp == 0) {
    // eq elements before each warp, then each warp's selected count and output offset
    const uint32_t gt = s_wa[lane], eq = s_wb[lane];
    uint32_t e_incl = eq;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, e_incl, o);
      if (lane >= o) e_incl += y;
    }
    const int64_t e_before = e_incl - eq;
    int64_t take = k_eq - e_before;
    take = take < 0 ? 0 : (take > eq ? eq : take);
    const int64_t lo = lane * chunk, hi = lo + chunk;
    const bool has_last = lo <= S - 1 && S - 1 < hi;
    int64_t sel = gt + take - (force && e_before == 0 && eq > 0 ? 1 : 0) + (force && has_last ? 1 : 0);
    uint32_t s_incl = static_cast<uint32_t>(sel);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s_incl, o);
      if (lane >= o) s_incl += y;
    }
    s_wa[lane] = static_cast<uint32_t>(e_before);
    s_wb[lane] = s_incl - static_cast<uint32_t>(sel);
    if (lane == 31 && s_incl != k) report(status, CBK_STATUS_COUNT);
  }
  __syncthreads();
  int64_t eq_rank0 = s_wa[warp], out = s_wb[warp];
  for (int64_t b0 = w_lo; b0 < w_hi; b0 += 32 * kTopkUnroll) {
  uint32_t keys[kTopkUnroll];
#pragma unroll
  for (int u = 0; u < kTopkUnroll; ++u) {
    const int64_t i = b0 + u * 32 + lane;
    keys[u] = i < w_hi ? key_at(i) : 0u;
  }
#pragma unroll
  for (int u = 0; u < kTopkUnroll; ++u) {
    const int64_t i = b0 + u * 32 + lane;
    const bool valid = i < w_hi;
    const uint32_t key = keys[u];
    const bool eq = valid && key == T;
    const unsigned eq_bal = __ballot_sync(0xffffffffu, eq);
    const int64_t eq_rank = eq_rank0 + __popc(eq_bal & lt_mask);
    bool sel = valid && (key > T || (eq && eq_rank < k_eq && !(force && eq_rank == 0)));
    if (force && valid && i == S - 1) sel = true;
    const unsigned sel_bal = __ballot_sync(0xffffffffu, sel);
    if (sel) {
      const int64_t at = out + __popc(sel_bal & lt_mask);
      if (at < k) idx[at] = i; else report(status, CBK_STATUS_COUNT);
    }
    eq_rank0 += __popc(eq_bal);
    out += __popc(sel_bal);
  }
  }
}

// Top-K for S <= kTopkSmallMax (blended prefills up to ~33K tokens): the
// same radix select and the same selection, with each thread holding a run of
// kTopkRun consecutive keys in registers (no shared-memory key array, no re-reads),
// and the ordered compaction as one block-wide scan of (keys above T, keys equal to
// T) per thread: a thread's first output slot is
//   (keys above T before it) + min(keys equal to T before it, k_eq)
//   - (1 if the last index is forced in and an equal key precedes it),
// since equal keys are ranked in index order and, when the last index is forced in,
// the equal key of rank 0 gives up its place.
constexpr int kTopkRunMax = 33;                                   // keys per thread, at most
constexpr int64_t kTopkSmallMax = int64_t{kTopkThreads} * kTopkRunMax;   // 33792

template <int kTopkRun>
__global__ void __launch_bounds__(kTopkThreads, 1)
topk_small_kernel(const float* __restrict__ dev, int64_t S64, int64_t k64, int force_last,
                  int64_t* __restrict__ idx, int32_t* status) {
  __shared__ uint32_t s_hist[256];
  __shared__ unsigned long long s_scan[kTopkWarps];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_krem, s_total_eq;
  const int S = static_cast<int>(S64), k = static_cast<int>(k64);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i0 = tid * kTopkRun;
  // launched as a programmatic dependent of the deviation kernel (a no-op otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int n_mine = min(max(S - i0, 0), kTopkRun);
  uint32_t key[kTopkRun];
#pragma unroll
  for (int r = 0; r < kTopkRun; ++r) key[r] = r < n_mine ? order_key(dev[i0 + r]) : 0u;
  const uint32_t last_key = order_key(dev[S - 1]);
  for (int b = tid; b < 256; b += kTopkThreads) s_hist[b] = 0;
  if (tid == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_krem = k;
  }
  __syncthreads();
  // four 8-bit radix passes, high digit first
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t prefix = s_prefix, mask = s_mask;
#pragma unroll
    for (int r = 0; r < kTopkRun; ++r)
      if (r < n_mine && (key[r] & mask) == prefix) atomicAdd(&s_hist[(key[r] >> shift) & 255u], 1u);
    __syncthreads();
    if (warp == 0) {
      // lane l sums the 8 digits 255-8l .. 248-8l (descending digit order)
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) { c[e] = s_hist[255 - 8 * lane - e]; sum += c[e]; }
#pragma unroll
      for (int e = 0; e < 8; ++e) s_hist[255 - 8 * lane - e] = 0;      // ready for the next pass
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const uint32_t excl = incl - sum;
      const int krem = s_krem;
      const bool here = (static_cast<int>(excl) < krem) && (static_cast<int>(incl) >= krem);
      const unsigned who = __ballot_sync(0xffffffffu, here);
      if (here && lane == __ffs(who) - 1) {
        uint32_t above = excl;
        for (int e = 0; e < 8; ++e) {
          if (static_cast<int>(above + c[e]) >= krem) {
            const uint32_t digit = 255 - 8 * lane - e;
            s_prefix = prefix | (digit << shift);
            s_mask = mask | (255u << shift);
            s_krem = krem - static_cast<int>(above);
            s_total_eq = static_cast<int>(c[e]);
            break;
          }
          above += c[e];
        }
      }
    }
    __syncthreads();
  }
  const uint32_t T = s_prefix;
  const int k_eq = s_krem, total_eq = s_total_eq;
  const bool last_sel = last_key > T || (last_key == T && total_eq <= k_eq);
  const bool force = force_last && !last_sel;
  // per-thread counts, one block-wide scan of (above, equal) packed in 64 bits
  uint32_t n_gt = 0, n_eq = 0;
#pragma unroll
  for (int r = 0; r < kTopkRun; ++r) {
    n_gt += (r < n_mine && key[r] > T) ? 1u : 0u;
    n_eq += (r < n_mine && key[r] == T) ? 1u : 0u;
  }
  const unsigned long long mine = (static_cast<unsigned long long>(n_gt) << 32) | n_eq;
  unsigned long long incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const unsigned long long w = s_scan[lane];
    unsigned long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    s_scan[lane] = wi - w;   // exclusive prefix of the warps' totals
    if (lane == 31) {
      // the selection's size: every key above T, k_eq equal ones, the forced last index
      const int gt_all = static_cast<int>(wi >> 32), eq_all = static_cast<int>(wi & 0xffffffffull);
      const int total = gt_all + min(eq_all, k_eq) + (force ? 1 : 0) - (force && eq_all > 0 ? 1 : 0);
      if (total != k) report(status, CBK_STATUS_COUNT);
    }
  }
  __syncthreads();
  const unsigned long long before = s_scan[warp] + incl - mine;
  const int gt_before = static_cast<int>(before >> 32), e_before = static_cast<int>(before & 0xffffffffull);
  int out = gt_before + min(e_before, k_eq) - (force && e_before > 0 ? 1 : 0);
  int eq_rank = e_before;
#pragma unroll
  for (int r = 0; r < kTopkRun; ++r) {
    if (r >= n_mine) break;
    const int i = i0 + r;
    const bool eq = key[r] == T;
    bool sel = key[r] > T || (eq && eq_rank < k_eq && !(force && eq_rank == 0));
    if (force && i == S - 1) sel = true;
    if (sel) {
      if (out < k) idx[out] = i; else report(status, CBK_STATUS_COUNT);
      ++out;
    }
    eq_rank += eq ? 1 : 0;
  }
}

int ensure_smem_attr(const void* func, int bytes);   // cbk_api.cu

static size_t topk_smem_bytes(int64_t S) {
  return S <= kTopkSmemKeys ? static_cast<size_t>(S) * sizeof(uint32_t) : 0;
}

static int launch_topk(const float* dev, int64_t S, int64_t k, int force_last, int64_t* idx,
                       int32_t* status, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kTopkThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see deviation_kernel
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (S <= kTopkSmallMax) {
    // keys per thread: 8, 16 or 33
    auto kern = S <= kTopkThreads * 8 ? topk_small_kernel<8>
                : S <= kTopkThreads * 16 ? topk_small_kernel<16> : topk_small_kernel<kTopkRunMax>;
    cfg.dynamicSmemBytes = 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, dev, S, k, force_last, idx, status);
    if (e != cudaSuccess) return set_error(CBK_ERR_CUDA, "topk_small_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("topk_small_kernel");
  }
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(topk_kernel),
                                static_cast<int>(kTopkSmemKeys * sizeof(uint32_t))))
    return rc;
  cfg.dynamicSmemBytes = topk_smem_bytes(S);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, topk_kernel, dev, S, k, force_last, idx, status);
  if (e != cudaSuccess) return set_error(CBK_ERR_CUDA, "topk_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("topk_kernel");
}

static int launch_deviation(const void* k_new, int64_t new_stride, const cbk_chunk_src* old_srcs,
                            const int64_t* chunk_start, int n_chunks, int64_t S, int64_t feat,
                            int dtype, float* dev, cudaStream_t st) {
  const int64_t blocks = (S * 32 + kDevThreads - 1) / kDevThreads;
  if (dtype == CBK_BF16)
    deviation_kernel<CBK_BF16><<<static_cast<unsigned>(blocks), kDevThreads, 0, st>>>(
        static_cast<const uint16_t*>(k_new), new_stride, old_srcs, chunk_start, n_chunks, S, feat, dev);
  else
    deviation_kernel<CBK_F16><<<static_cast<unsigned>(blocks), kDevThreads, 0, st>>>(
        static_cast<const uint16_t*>(k_new), new_stride, old_srcs, chunk_start, n_chunks, S, feat, dev);
  return check_launch("deviation_kernel");
}

static int check_dev_args(const char* fn, const void* k_new, int64_t new_stride,
                          const cbk_chunk_src* old_srcs, const int64_t* chunk_start, int n_chunks,
                          int64_t S, int64_t feat, int dtype) {
  if (dtype != CBK_BF16 && dtype != CBK_F16)
    return set_error(CBK_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16/fp16 only)", fn, dtype);
  if (!k_new || !old_srcs || !chunk_start)
    return set_error(CBK_ERR_INVALID, "%s: null pointer argument", fn);
  if (S <= 0 || n_chunks <= 0 || feat <= 0 || feat % 8 != 0 || feat >= kDevMaxFeat || new_stride < feat ||
      new_stride % 8)
    return set_error(CBK_ERR_INVALID, "%s: bad sizes (S %lld, chunks %d, feat %lld, stride %lld)",
                     fn, (long long)S, n_chunks, (long long)feat, (long long)new_stride);
  if (reinterpret_cast<uintptr_t>(k_new) & 15u)
    return set_error(CBK_ERR_INVALID, "%s: K_new must be 16-byte aligned", fn);
  return CBK_OK;
}

}  // namespace cbk

using namespace cbk;

extern "C" int cbk_kv_deviation(const void* k_new, int64_t new_row_stride,
                                const cbk_chunk_src* old_srcs, const int64_t* chunk_start,
                                int n_chunks, int64_t S, int64_t feat, int dtype, float* dev,
                                void* stream) {
  if (int rc = check_dev_args("cbk_kv_deviation", k_new, new_row_stride, old_srcs, chunk_start,
                              n_chunks, S, feat, dtype))
    return rc;
  if (!dev) return set_error(CBK_ERR_INVALID, "cbk_kv_deviation: null output");
  return launch_deviation(k_new, new_row_stride, old_srcs, chunk_start, n_chunks, S, feat, dtype,
                          dev, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t cbk_topk_count(int64_t S, double ratio) {
  int64_t k = static_cast<int64_t>(static_cast<double>(S) * ratio);   // truncation, like int()
  if (k < 1) k = 1;
  if (k > S) k = S;
  return k;
}

extern "C" int cbk_topk_select(const float* dev, int64_t S, int64_t k, int force_last,
                               int64_t* idx, int32_t* status, void* stream) {
  if (!dev || !idx) return set_error(CBK_ERR_INVALID, "cbk_topk_select: null pointer argument");
  if (S <= 0 || k <= 0 || k > S)
    return set_error(CBK_ERR_INVALID, "cbk_topk_select: need 0 < k <= S (k %lld, S %lld)",
                     (long long)k, (long long)S);
  return launch_topk(dev, S, k, force_last, idx, status, static_cast<cudaStream_t>(stream));
}

extern "C" size_t cbk_hkvd_workspace_bytes(int64_t S) {
  return S <= 0 ? 0 : ((static_cast<size_t>(S) * sizeof(float) + 255) / 256) * 256;
}

extern "C" int cbk_hkvd_select(const void* k_new, int64_t new_row_stride,
                               const cbk_chunk_src* old_srcs, const int64_t* chunk_start,
                               int n_chunks, int64_t S, int64_t feat, int dtype, int64_t k,
                               int force_last, int64_t* idx, void* workspace,
                               size_t workspace_bytes, int32_t* status, void* stream) {
  if (int rc = check_dev_args("cbk_hkvd_select", k_new, new_row_stride, old_srcs, chunk_start,
                              n_chunks, S, feat, dtype))
    return rc;
  if (!idx || !workspace) return set_error(CBK_ERR_INVALID, "cbk_hkvd_select: null output/workspace");
  if (k <= 0 || k > S) return set_error(CBK_ERR_INVALID, "cbk_hkvd_select: need 0 < k <= S");
  if (workspace_bytes < cbk_hkvd_workspace_bytes(S))
    return set_error(CBK_ERR_WORKSPACE, "cbk_hkvd_select: workspace %zu < %zu bytes", workspace_bytes,
                     cbk_hkvd_workspace_bytes(S));
  auto st = static_cast<cudaStream_t>(stream);
  float* dev = static_cast<float*>(workspace);
  if (int rc = launch_deviation(k_new, new_row_stride, old_srcs, chunk_start, n_chunks, S, feat,
                                dtype, dev, st))
    return rc;
  return launch_topk(dev, S, k, force_last, idx, status, st);
}

// ---------------------------------------------------------------------------
// HKVD selection without any allocation.
//
// Some callers cannot allocate device memory at the moment they select tokens:
// a serving engine that reserves nearly all HBM for its own KV-cache pool up
// front (an extra cudaMalloc then fails or fragments that pool), or a
// latency-critical step where cudaMalloc / cudaFree would synchronise the
// device.  For them the deviation scores live in a fixed scratch array that the
// library owns: kNoAllocMaxTokens fp32 (1 MiB) in device memory, held on every
// GPU that loads the library until the process exits.
//
// The array's host-side name is only a stand-in for the device address, so the
// address is looked up with cudaGetSymbolAddress once per device, on the first
// call made with that device current, and kept for the process; make that
// first call before any stream capture.  A device reset (cudaDeviceReset or a
// primary-context reset) reloads the module and may move the array, leaving
// the kept address stale: the entry point is not for use after a reset.  All calls share the array and it keeps the previous call's
// contents; nothing in it is read before this call writes it (positions
// [0, S) are written by the deviation kernel before the top-K kernel reads
// them), so nothing needs clearing.  Calls that overlap on the GPU (two streams,
// or two threads on different streams of one device) race on the array: order
// them on one stream.
// ---------------------------------------------------------------------------
namespace cbk {

constexpr int64_t kNoAllocMaxTokens = 262144;
static __device__ __align__(256) float g_hkvd_noalloc_scratch[kNoAllocMaxTokens];

static int noalloc_scratch(float** out) {
  static std::mutex mu;
  static float* addr[64] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(CBK_ERR_CUDA, "cbk_hkvd_select_noalloc: cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_hkvd_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(CBK_ERR_CUDA, "cbk_hkvd_select_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return CBK_OK;
}

}  // namespace cbk

extern "C" int64_t cbk_hkvd_noalloc_max_tokens(void) { return kNoAllocMaxTokens; }

extern "C" int cbk_hkvd_select_noalloc(const void* k_new, int64_t new_row_stride,
                                       const cbk_chunk_src* old_srcs, const int64_t* chunk_start,
                                       int n_chunks, int64_t S, int64_t feat, int dtype, int64_t k,
                                       int force_last, int64_t* idx, int32_t* status, void* stream) {
  if (int rc = check_dev_args("cbk_hkvd_select_noalloc", k_new, new_row_stride, old_srcs,
                              chunk_start, n_chunks, S, feat, dtype))
    return rc;
  if (!idx) return set_error(CBK_ERR_INVALID, "cbk_hkvd_select_noalloc: null output");
  if (S > kNoAllocMaxTokens)
    return set_error(CBK_ERR_INVALID,
                     "cbk_hkvd_select_noalloc: S = %lld tokens exceeds the fixed scratch of %lld "
                     "tokens; use cbk_hkvd_select with a caller workspace",
                     (long long)S, (long long)kNoAllocMaxTokens);
  if (k <= 0 || k > S) return set_error(CBK_ERR_INVALID, "cbk_hkvd_select_noalloc: need 0 < k <= S");
  float* dev = nullptr;
  if (int rc = noalloc_scratch(&dev)) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  if (int rc = launch_deviation(k_new, new_row_stride, old_srcs, chunk_start, n_chunks, S, feat,
                                dtype, dev, st))
    return rc;
  return launch_topk(dev, S, k, force_last, idx, status, st);
}
