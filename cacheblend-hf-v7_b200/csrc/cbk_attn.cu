// Partial-query attention on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA computes a 128-row tile of (selected token, q-head) rows that share
// one KV head: rows r = tok * G + h (G = q heads per KV head), TOK = 128 / G
// selected tokens.  Keys are visited in 128-key tiles from 0 up to the largest
// position in the tile; causality is a per-row position compare (no mask
// tensor).  Accumulators live in TMEM: S = Q K^T (128 fp32 columns) and
// O = P V (head_dim fp32 columns).
//
// Warp roles (256 threads):
//   warp 0      TMA producer: Q once, then K/V tiles into a 2-stage ring
//   warp 1      MMA issuer:   S(j+1) = Q K(j+1)^T is issued before O += P(j) V(j)
//   warp 2      TMEM allocator
//   warps 4..7  softmax + epilogue: thread i of warp w owns TMEM lane
//               32*(w%4)+i, i.e. one full row; row max / exp / sum are
//               thread-local.  O is rescaled only when the running max grows
//               by more than 2^8 (the final O / l uses the same stale max).
// Every mbarrier wait is bounded (2 s of wall time); on timeout the kernel
// sets CBK_STATUS_TIMEOUT, drains its own TMA copies and MMAs, frees TMEM and
// returns.
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "cbk_common.cuh"

namespace cbk {

constexpr int kBM = 128;       // rows per CTA tile
constexpr int kBN = 128;       // keys per KV tile
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 256;

template <int HD>
struct AttnSmem {
  static constexpr int kQBytes = kBM * HD * 2;
  static constexpr int kKVBytes = kBN * HD * 2;
  static constexpr int kPBytes = kBM * kBN * 2;
  static constexpr int kQ = 0;
  static constexpr int kK0 = kQ + kQBytes;
  static constexpr int kV0 = kK0 + 2 * kKVBytes;
  static constexpr int kP = kV0 + 2 * kKVBytes;
  static constexpr int kBar = kP + kPBytes;            // 16 x 8-byte barriers
  static constexpr int kMisc = kBar + 16 * 8;          // tmem slot + abort flag
  static constexpr int kTotal = kMisc + 16;
  static constexpr int kAlloc = kTotal + 1024;         // slack for 1024-byte alignment
};

enum Bar { B_Q = 0, B_KVFULL0 = 1, B_KVEMPTY0 = 3, B_SFULL = 5, B_SFREE = 6, B_PFULL = 7,
           B_ODONE = 8, B_DRAIN = 9 };

struct AttnParams {
  const int64_t* pos;
  uint16_t* out;
  int32_t* status;
  int64_t n_sel;
  int n_q_heads;
  int group;          // G
  int tok_per_tile;   // 128 / G
  int n_tiles;
  float scale_log2;
};

__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

template <int DT, int HD>
__global__ void __launch_bounds__(kThreads, 1)
partial_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const AttnParams prm) {
  using L = AttnSmem<HD>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - raw_addr);
  const uint32_t sQ = base + L::kQ, sK0 = base + L::kK0, sV0 = base + L::kV0, sP = base + L::kP;
  auto bar = [&](int i) { return base + L::kBar + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sbase + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sbase + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = prm.n_tiles - 1 - static_cast<int>(blockIdx.x);   // longest tiles first
  const int kvh = blockIdx.y;
  const int64_t tok0 = static_cast<int64_t>(tile) * prm.tok_per_tile;
  const int64_t tok_end = min(tok0 + prm.tok_per_tile, prm.n_sel);
  const int64_t p_max = prm.pos[tok_end - 1];
  const int n_kv = static_cast<int>(p_max / kBN) + 1;

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    mbar_init(bar(B_KVFULL0), 1);
    mbar_init(bar(B_KVFULL0 + 1), 1);
    mbar_init(bar(B_KVEMPTY0), 1);
    mbar_init(bar(B_KVEMPTY0 + 1), 1);
    mbar_init(bar(B_SFULL), 1);
    mbar_init(bar(B_SFREE), 4);
    mbar_init(bar(B_PFULL), 4);
    mbar_init(bar(B_ODONE), 1);
    mbar_init(bar(B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + kBN;
  bool failed = false;

  if (warp == 0 && lane == 0) {
    // ----------------------------------------------------------- TMA producer
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    mbar_expect_tx(bar(B_Q), L::kQBytes);
#pragma unroll
    for (int h = 0; h < HD / 64; ++h)
      tma_load_3d(sQ + h * (kBM * 128), &tm_q, bar(B_Q), h * 64, kvh * prm.group,
                  static_cast<int>(tok0));
    int last_armed[2] = {-1, -1};
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      if (j >= 2 && !wait_or_abort(bar(B_KVEMPTY0 + st), ((j >> 1) - 1) & 1, abort_flag)) {
        failed = true;
        break;
      }
      mbar_expect_tx(bar(B_KVFULL0 + st), 2 * L::kKVBytes);
      const uint32_t dk = sK0 + st * L::kKVBytes, dv = sV0 + st * L::kKVBytes;
#pragma unroll
      for (int h = 0; h < HD / 64; ++h) {
        tma_load_3d(dk + h * (kBN * 128), &tm_k, bar(B_KVFULL0 + st), h * 64, kvh, j * kBN);
        tma_load_3d(dv + h * (kBN * 128), &tm_v, bar(B_KVFULL0 + st), h * 64, kvh, j * kBN);
      }
      last_armed[st] = j;
    }
    // Drain: every armed copy must land before the CTA can retire.
    if (!mbar_wait(bar(B_Q), 0)) failed = true;
    for (int st = 0; st < 2; ++st)
      if (last_armed[st] >= 0 && !mbar_wait(bar(B_KVFULL0 + st), (last_armed[st] >> 1) & 1))
        failed = true;
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------- MMA issuer
    const uint32_t idesc_s = umma_idesc_f16(DT, kBM, kBN, 0);
    const uint32_t idesc_o = umma_idesc_f16(DT, kBM, HD, 1);
    auto issue_s = [&](int j) {
      const int st = j & 1;
      const uint32_t kb = sK0 + st * L::kKVBytes;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint32_t off = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
        const uint32_t offk = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
        umma_f16_ss(tS, umma_desc_sw128(sQ + off, 16, 1024), umma_desc_sw128(kb + offk, 16, 1024),
                    idesc_s, kk > 0 ? 1u : 0u);
      }
      umma_commit(bar(B_SFULL));
    };
    do {
      if (!wait_or_abort(bar(B_Q), 0, abort_flag) ||
          !wait_or_abort(bar(B_KVFULL0), 0, abort_flag)) { failed = true; break; }
      tc_fence_after();
      issue_s(0);
      for (int j = 0; j < n_kv; ++j) {
        if (j + 1 < n_kv) {
          const int st1 = (j + 1) & 1;
          if (!wait_or_abort(bar(B_KVFULL0 + st1), ((j + 1) >> 1) & 1, abort_flag) ||
              !wait_or_abort(bar(B_SFREE), j & 1, abort_flag)) { failed = true; break; }
          tc_fence_after();
          issue_s(j + 1);
        }
        if (!wait_or_abort(bar(B_PFULL), j & 1, abort_flag)) { failed = true; break; }
        tc_fence_after();
        const uint32_t vb = sV0 + (j & 1) * L::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t offp = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          umma_f16_ss(tO, umma_desc_sw128(sP + offp, 16, 1024),
                      umma_desc_sw128(vb + kk * 16 * 128, kBN * 128, 1024), idesc_o,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar(B_ODONE));
        umma_commit(bar(B_KVEMPTY0 + (j & 1)));
      }
    } while (false);
    // Drain: all MMAs issued by this thread complete before TMEM is released.
    umma_commit(bar(B_DRAIN));
    if (!mbar_wait(bar(B_DRAIN), 0)) failed = true;
  } else if (warp >= 4) {
    // ----------------------------------------------- softmax + epilogue warps
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int64_t tok = tok0 + row / prm.group;
    const bool row_valid = tok < tok_end;
    const int64_t p_row = row_valid ? prm.pos[tok] : p_max;
    float m_used = -INFINITY, l_sum = 0.f;
    const float sl2 = prm.scale_log2;
    uint8_t* prow = sbase + L::kP + row * 128;
    for (int j = 0; j < n_kv; ++j) {
      if (!__all_sync(0xffffffffu, wait_or_abort(bar(B_SFULL), j & 1, abort_flag))) {
        failed = true;
        break;
      }
      tc_fence_after();
      uint32_t s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c)
        tmem_ld32(tS + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_SFREE));
      // causal limit inside this tile: keys j*kBN + c valid iff <= p_row
      const int64_t lim64 = p_row - static_cast<int64_t>(j) * kBN;
      const int lim = lim64 >= kBN ? kBN : static_cast<int>(lim64);   // keys c <= lim are visible
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBN; ++c)
        if (c <= lim) mx = fmaxf(mx, __uint_as_float(s[c]));
      const float m_tile = mx * sl2;
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_used = m_tile;
      } else if (m_tile > m_used + 8.f) {
        alpha = ex2(m_used - m_tile);
        m_used = m_tile;
        rescale = true;
      }
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kBN; ++c) {
        const float p = (c <= lim) ? ex2(__uint_as_float(s[c]) * sl2 - m_used) : 0.f;
        s[c] = __float_as_uint(p);
        rs += p;
      }
      l_sum = l_sum * alpha + rs;
      if (j > 0) {
        if (!__all_sync(0xffffffffu, wait_or_abort(bar(B_ODONE), (j - 1) & 1, abort_flag))) {
          failed = true;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + lane_off + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + lane_off + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      // P (16-bit) into the K-major, 128-byte-swizzled operand tile
#pragma unroll
      for (int ch = 0; ch < kBN / 8; ++ch) {
        uint4 v;
        uint16_t* h = reinterpret_cast<uint16_t*>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = Elem<DT>::from_f(__uint_as_float(s[ch * 8 + e]));
        const int sub_tile = ch >> 3, cc = ch & 7;
        *reinterpret_cast<uint4*>(prow + sub_tile * (kBM * 128) + ((cc ^ (row & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PFULL));
    }
    if (!failed) {
      if (!__all_sync(0xffffffffu, wait_or_abort(bar(B_ODONE), (n_kv - 1) & 1, abort_flag))) {
        failed = true;
      } else {
        tc_fence_after();
        const float inv_l = 1.f / l_sum;
        const int hq = kvh * prm.group + row % prm.group;
        uint16_t* orow = prm.out + (tok * prm.n_q_heads + hq) * static_cast<int64_t>(HD);
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + lane_off + c * 32, o);
          tmem_wait_ld();
          if (row_valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 v;
              uint16_t* h = reinterpret_cast<uint16_t*>(&v);
#pragma unroll
              for (int e = 0; e < 8; ++e) h[e] = Elem<DT>::from_f(__uint_as_float(o[q * 8 + e]) * inv_l);
              st_vec(orow + c * 32 + q * 8, v);
            }
          }
        }
      }
    }
  }

  if (failed) {
    *abort_flag = 1;
    report(prm.status, CBK_STATUS_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side: tensor maps + launch
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D map over [d2][d1][d0] 16-bit elements, box {64, b1, b2}, 128-byte swizzle.
static int make_map(CUtensorMap* m, const void* ptr, int dtype, uint64_t d0, uint64_t d1, uint64_t d2,
                    uint32_t b1, uint32_t b2) {
  auto enc = get_encode_fn();
  if (!enc) return set_error(CBK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  const cuuint32_t box[3] = {64, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, dtype == CBK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         3, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(CBK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CBK_OK;
}

int ensure_smem_attr(const void* func, int bytes);   // cbk_api.cu

template <int DT, int HD>
static int launch_attn(const void* q, const void* k, const void* v, const int64_t* pos,
                       int64_t n_sel, int64_t S, int n_q_heads, int n_kv_heads, float scale,
                       void* out, int32_t* status, cudaStream_t st) {
  const int G = n_q_heads / n_kv_heads;
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, q, DT, HD, n_q_heads, n_sel, G, kBM / G)) return rc;
  if (int rc = make_map(&mk, k, DT, HD, n_kv_heads, S, 1, kBN)) return rc;
  if (int rc = make_map(&mv, v, DT, HD, n_kv_heads, S, 1, kBN)) return rc;
  AttnParams prm;
  prm.pos = pos;
  prm.out = static_cast<uint16_t*>(out);
  prm.status = status;
  prm.n_sel = n_sel;
  prm.n_q_heads = n_q_heads;
  prm.group = G;
  prm.tok_per_tile = kBM / G;
  prm.n_tiles = static_cast<int>((n_sel + prm.tok_per_tile - 1) / prm.tok_per_tile);
  prm.scale_log2 = scale * 1.4426950408889634f;
  auto kern = partial_attn_kernel<DT, HD>;
  const int smem = AttnSmem<HD>::kAlloc;
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem)) return rc;
  dim3 grid(static_cast<unsigned>(prm.n_tiles), static_cast<unsigned>(n_kv_heads));
  kern<<<grid, kThreads, smem, st>>>(mq, mk, mv, prm);
  return check_launch("partial_attn_kernel");
}

}  // namespace cbk

using namespace cbk;

extern "C" int cbk_partial_attn(const void* q, const void* k, const void* v, const int64_t* pos,
                                int64_t n_sel, int64_t S, int n_q_heads, int n_kv_heads,
                                int head_dim, float scale, int dtype, void* out, int32_t* status,
                                void* stream) {
  if (dtype != CBK_BF16 && dtype != CBK_F16)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_partial_attn: dtype %d not supported", dtype);
  if (head_dim != 64 && head_dim != 128)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_partial_attn: head_dim %d (64 or 128 only)", head_dim);
  if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads != 0)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: n_q_heads must be a multiple of n_kv_heads");
  const int G = n_q_heads / n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_partial_attn: GQA group %d not in {1,2,4,8,16}", G);
  if (!q || !k || !v || !pos || !out)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: null pointer argument");
  if (S <= 0 || n_sel < 0 || S > (int64_t(1) << 31) || n_sel > (int64_t(1) << 31))
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: bad sizes");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: q/k/v/out must be 16-byte aligned");
  if ((n_sel + (128 / G) - 1) / (128 / G) > 2147483647LL)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: too many tiles");
  if (n_sel == 0) return CBK_OK;
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == CBK_BF16)
    return head_dim == 128
               ? launch_attn<CBK_BF16, 128>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, status, st)
               : launch_attn<CBK_BF16, 64>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, status, st);
  return head_dim == 128
             ? launch_attn<CBK_F16, 128>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, status, st)
             : launch_attn<CBK_F16, 64>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, status, st);
}
