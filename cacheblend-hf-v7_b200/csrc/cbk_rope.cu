// RoPE table, chunk-KV assembly (concat + RoPE shift), row RoPE and the
// per-layer fresh-row RoPE + scatter.  All of these are HBM-bound byte movers:
// 128-bit loads/stores, one pass over the data, rotation in fp32 registers.
#include "cbk_common.cuh"

namespace cbk {

// ---------------------------------------------------------------------------
// cos/sin table: one thread per (position, frequency).
// Angle = fp32(inv_freq[i]) * fp32(p), as MistralRotaryEmbedding.forward
// computes it (the K=1 matmul of inv_freq by position_ids is one rounded
// product); cos/sin evaluated in fp32 and scaled by attention_scaling.
// ---------------------------------------------------------------------------
__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int half_dim, int64_t n_pos,
                                  float scaling, float2* __restrict__ table) {
  const int64_t n = n_pos * half_dim;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = e / half_dim;
    const int i = static_cast<int>(e - p * half_dim);
    const float ang = __fmul_rn(inv_freq[i], static_cast<float>(p));
    table[e] = make_float2(__fmul_rn(cosf(ang), scaling), __fmul_rn(sinf(ang), scaling));
  }
}

// ---------------------------------------------------------------------------
// Rotate 8 (lo, hi) element pairs of one head:
//   out_lo = x_lo * cos - x_hi * sin,  out_hi = x_hi * cos + x_lo * sin
// (rotate_half layout: element j pairs with j + D/2, both use frequency j).
// CBK_ROPE_REF reproduces the 16-bit torch op sequence of apply_rotary_pos_emb:
// cos/sin rounded to the element type, each product rounded, the sum rounded.
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void rope8(const uint4& lo, const uint4& hi, const float2* cs,
                                      int mode, uint4& olo, uint4& ohi) {
  const uint16_t* xl = reinterpret_cast<const uint16_t*>(&lo);
  const uint16_t* xh = reinterpret_cast<const uint16_t*>(&hi);
  uint16_t* yl = reinterpret_cast<uint16_t*>(&olo);
  uint16_t* yh = reinterpret_cast<uint16_t*>(&ohi);
  // table entries for 8 consecutive frequencies: 4 x 16-byte loads
  float2 t[8];
  const float4* c4 = reinterpret_cast<const float4*>(cs);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = c4[q];
    t[2 * q] = make_float2(v.x, v.y);
    t[2 * q + 1] = make_float2(v.z, v.w);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a = Elem<DT>::to_f(xl[e]);
    const float b = Elem<DT>::to_f(xh[e]);
    float c = t[e].x, s = t[e].y;
    if (mode == CBK_ROPE_REF) {
      c = round16<DT>(c);
      s = round16<DT>(s);
      const float ac = round16<DT>(__fmul_rn(a, c));
      const float bs = round16<DT>(__fmul_rn(b, s));
      const float bc = round16<DT>(__fmul_rn(b, c));
      const float as = round16<DT>(__fmul_rn(a, s));
      yl[e] = Elem<DT>::from_f(__fadd_rn(ac, -bs));
      yh[e] = Elem<DT>::from_f(__fadd_rn(bc, as));
    } else {
      yl[e] = Elem<DT>::from_f(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)));
      yh[e] = Elem<DT>::from_f(__fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s)));
    }
  }
}

// Rotate one 8-pair group (head h, pair group g) of a row and store it.
template <int DT, bool STREAM>
__device__ __forceinline__ void rope_group(const uint16_t* src_row, uint16_t* dst_row, int h, int g,
                                           int head_dim, const float2* cs_row, int mode) {
  const int half = head_dim >> 1;
  const int off = h * head_dim + g * 8;
  const uint4 lo = STREAM ? ld_stream(src_row + off) : ld_vec(src_row + off);
  const uint4 hi = STREAM ? ld_stream(src_row + off + half) : ld_vec(src_row + off + half);
  uint4 olo, ohi;
  rope8<DT>(lo, hi, cs_row + g * 8, mode, olo, ohi);
  st_vec(dst_row + off, olo);
  st_vec(dst_row + off + half, ohi);
}

// ---------------------------------------------------------------------------
// (a)+(b) assemble: rows of one layer per blockIdx.y, kRows rows per block.
// Work items of a row: n_kv_heads * head_dim/16 K pair-groups (RoPE) followed
// by kv_dim/8 V vectors (copy).
// ---------------------------------------------------------------------------
constexpr int kAsmThreads = 256;
constexpr int kAsmRows = 16;
constexpr int kMaxChunksSmem = 2048;

template <int DT>
__global__ void __launch_bounds__(kAsmThreads)
assemble_kernel(const cbk_chunk_src* __restrict__ srcs, const int64_t* __restrict__ chunk_start,
                int n_chunks, int64_t S, int n_kv_heads, int head_dim,
                const float2* __restrict__ table, int64_t table_rows,
                const int64_t* __restrict__ positions, int mode, uint16_t* __restrict__ k_out,
                uint16_t* __restrict__ v_out, int64_t layer_stride, int32_t* status) {
  __shared__ int64_t s_start[kMaxChunksSmem + 1];
  const int layer = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kAsmRows;
  for (int c = threadIdx.x; c <= n_chunks; c += blockDim.x) s_start[c] = chunk_start[c];
  __syncthreads();

  const int kv_dim = n_kv_heads * head_dim;
  const int kgroups = n_kv_heads * (head_dim >> 4);   // K pair-groups per row
  const int vvecs = kv_dim >> 3;                       // V 16-byte vectors per row
  const int per_row = kgroups + vvecs;
  const int n_items = kAsmRows * per_row;
  const cbk_chunk_src* lsrc = srcs + static_cast<int64_t>(layer) * n_chunks;
  uint16_t* kl = k_out + layer * layer_stride;
  uint16_t* vl = v_out + layer * layer_stride;

  for (int it = threadIdx.x; it < n_items; it += kAsmThreads) {
    const int r = it / per_row;
    const int w = it - r * per_row;
    const int64_t t = row0 + r;
    if (t >= S) continue;
    // chunk of row t: largest c with s_start[c] <= t
    int lo = 0, hi = n_chunks - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_start[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int64_t local = t - s_start[lo];
    if (w < kgroups) {
      const int64_t p = positions ? positions[t] : t;
      if (p < 0 || p >= table_rows) { report(status, CBK_STATUS_BAD_INDEX); continue; }
      const int h = w / (head_dim >> 4);
      const int g = w - h * (head_dim >> 4);
      const uint16_t* src = static_cast<const uint16_t*>(lsrc[lo].k) + local * kv_dim;
      rope_group<DT, true>(src, kl + t * kv_dim, h, g, head_dim, table + p * (head_dim >> 1), mode);
    } else {
      const int vv = w - kgroups;
      const uint16_t* src = static_cast<const uint16_t*>(lsrc[lo].v) + local * kv_dim + vv * 8;
      st_vec(vl + t * kv_dim + vv * 8, ld_stream(src));
    }
  }
}

// ---------------------------------------------------------------------------
// RoPE on plain rows with explicit positions (apply_rope_shift).
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256)
rope_rows_kernel(const uint16_t* in, uint16_t* out, int64_t n_rows, int n_heads, int head_dim,
                 const float2* __restrict__ table, int64_t table_rows,
                 const int64_t* __restrict__ positions, int mode, int32_t* status) {
  const int groups = n_heads * (head_dim >> 4);
  const int64_t n = n_rows * groups;
  const int row_elems = n_heads * head_dim;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / groups;
    const int w = static_cast<int>(e - r * groups);
    const int64_t p = positions[r];
    if (p < 0 || p >= table_rows) { report(status, CBK_STATUS_BAD_INDEX); continue; }
    const int h = w / (head_dim >> 4);
    const int g = w - h * (head_dim >> 4);
    rope_group<DT, false>(in + r * row_elems, out + r * row_elems, h, g, head_dim,
                          table + p * (head_dim >> 1), mode);
  }
}

// ---------------------------------------------------------------------------
// Fresh rows of one layer: RoPE(Q) -> q_out, RoPE(K) and V scattered into the
// fused cache at the selected positions.  Items per selected row j:
// Hq*D/16 Q groups, Hkv*D/16 K groups, Hkv*D/8 V vectors.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256)
rope_scatter_kernel(const uint16_t* __restrict__ q_src, int64_t q_stride,
                    const uint16_t* __restrict__ k_src, int64_t k_stride,
                    const uint16_t* __restrict__ v_src, int64_t v_stride, int gather,
                    const int64_t* __restrict__ idx, int64_t n_sel, int64_t S, int n_q_heads,
                    int n_kv_heads, int head_dim, const float2* __restrict__ table,
                    int64_t table_rows, int mode, uint16_t* __restrict__ q_out,
                    uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache,
                    int32_t* status) {
  const int gpr = head_dim >> 4;
  const int qg = n_q_heads * gpr;
  const int kg = n_kv_heads * gpr;
  const int kv_dim = n_kv_heads * head_dim;
  const int vv = kv_dim >> 3;
  const int per = qg + kg + vv;
  const int64_t n = n_sel * per;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e / per;
    int w = static_cast<int>(e - j * per);
    const int64_t p = idx[j];
    if (p < 0 || p >= S || p >= table_rows) { report(status, CBK_STATUS_BAD_INDEX); continue; }
    const int64_t r = gather ? p : j;
    const float2* cs = table + p * (head_dim >> 1);
    if (w < qg) {
      const int h = w / gpr, g = w - (w / gpr) * gpr;
      rope_group<DT, false>(q_src + r * q_stride, q_out + j * (int64_t)(n_q_heads * head_dim), h, g,
                            head_dim, cs, mode);
    } else if ((w -= qg) < kg) {
      const int h = w / gpr, g = w - (w / gpr) * gpr;
      rope_group<DT, false>(k_src + r * k_stride, k_cache + p * kv_dim, h, g, head_dim, cs, mode);
    } else {
      w -= kg;
      st_vec(v_cache + p * kv_dim + w * 8, ld_vec(v_src + r * v_stride + w * 8));
    }
  }
}

static int grid_for(int64_t items, int threads, int max_blocks = 148 * 16) {
  int64_t b = (items + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return static_cast<int>(b);
}

}  // namespace cbk

using namespace cbk;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int cbk_rope_table(const float* inv_freq, int half_dim, int64_t n_pos,
                              float attention_scaling, void* table, void* stream) {
  if (!inv_freq || !table || half_dim <= 0 || n_pos <= 0)
    return set_error(CBK_ERR_INVALID, "cbk_rope_table: null pointer or empty size");
  const int64_t n = n_pos * half_dim;
  rope_table_kernel<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      inv_freq, half_dim, n_pos, attention_scaling, static_cast<float2*>(table));
  return check_launch("rope_table_kernel");
}

static int check_mode(const char* fn, int rope_mode) {
  if (rope_mode != CBK_ROPE_REF && rope_mode != CBK_ROPE_FP32)
    return set_error(CBK_ERR_INVALID, "%s: bad rope_mode %d", fn, rope_mode);
  return CBK_OK;
}

static int check_geometry(const char* fn, int n_heads, int head_dim, int dtype) {
  if (dtype != CBK_BF16 && dtype != CBK_F16)
    return set_error(CBK_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16/fp16 only)", fn, dtype);
  if (head_dim <= 0 || head_dim % 16 != 0 || head_dim > 256)
    return set_error(CBK_ERR_UNSUPPORTED, "%s: head_dim %d must be a multiple of 16 <= 256", fn,
                     head_dim);
  if (n_heads <= 0) return set_error(CBK_ERR_INVALID, "%s: n_heads must be positive", fn);
  return CBK_OK;
}

extern "C" int cbk_assemble_kv(const cbk_chunk_src* srcs, const int64_t* chunk_start, int n_chunks,
                               int n_layers, int64_t S, int n_kv_heads, int head_dim, int dtype,
                               const void* rope_table, int64_t table_rows,
                               const int64_t* positions, int rope_mode, void* k_out, void* v_out,
                               int64_t out_layer_stride, int32_t* status, void* stream) {
  if (int rc = check_geometry("cbk_assemble_kv", n_kv_heads, head_dim, dtype)) return rc;
  if (!srcs || !chunk_start || !rope_table || !k_out || !v_out)
    return set_error(CBK_ERR_INVALID, "cbk_assemble_kv: null pointer argument");
  if (n_chunks <= 0 || n_chunks > kMaxChunksSmem || n_layers <= 0 || S <= 0)
    return set_error(CBK_ERR_INVALID, "cbk_assemble_kv: bad sizes (chunks %d, layers %d, S %lld)",
                     n_chunks, n_layers, (long long)S);
  if (n_layers > 65535) return set_error(CBK_ERR_INVALID, "cbk_assemble_kv: too many layers");
  if (!aligned16(k_out) || !aligned16(v_out) || !aligned16(rope_table) ||
      out_layer_stride % 8 != 0 || out_layer_stride < S * n_kv_heads * head_dim)
    return set_error(CBK_ERR_INVALID, "cbk_assemble_kv: outputs must be 16-byte aligned with a layer "
                     "stride >= S*kv_dim (multiple of 8)");
  if (int rc = check_mode("cbk_assemble_kv", rope_mode)) return rc;
  dim3 grid(static_cast<unsigned>((S + kAsmRows - 1) / kAsmRows), static_cast<unsigned>(n_layers));
  auto st = static_cast<cudaStream_t>(stream);
  auto tab = static_cast<const float2*>(rope_table);
  if (dtype == CBK_BF16)
    assemble_kernel<CBK_BF16><<<grid, kAsmThreads, 0, st>>>(
        srcs, chunk_start, n_chunks, S, n_kv_heads, head_dim, tab, table_rows, positions, rope_mode,
        static_cast<uint16_t*>(k_out), static_cast<uint16_t*>(v_out), out_layer_stride, status);
  else
    assemble_kernel<CBK_F16><<<grid, kAsmThreads, 0, st>>>(
        srcs, chunk_start, n_chunks, S, n_kv_heads, head_dim, tab, table_rows, positions, rope_mode,
        static_cast<uint16_t*>(k_out), static_cast<uint16_t*>(v_out), out_layer_stride, status);
  return check_launch("assemble_kernel");
}

extern "C" int cbk_rope_rows(const void* in, void* out, int64_t n_rows, int n_heads, int head_dim,
                             int dtype, const void* rope_table, int64_t table_rows,
                             const int64_t* positions, int rope_mode, int32_t* status,
                             void* stream) {
  if (int rc = check_geometry("cbk_rope_rows", n_heads, head_dim, dtype)) return rc;
  if (int rc = check_mode("cbk_rope_rows", rope_mode)) return rc;
  if (!in || !out || !rope_table || !positions)
    return set_error(CBK_ERR_INVALID, "cbk_rope_rows: null pointer argument");
  if (n_rows < 0) return set_error(CBK_ERR_INVALID, "cbk_rope_rows: negative row count");
  if (!aligned16(in) || !aligned16(out) || !aligned16(rope_table))
    return set_error(CBK_ERR_INVALID, "cbk_rope_rows: buffers must be 16-byte aligned");
  if (n_rows == 0) return CBK_OK;
  const int64_t items = n_rows * n_heads * (head_dim >> 4);
  auto st = static_cast<cudaStream_t>(stream);
  auto tab = static_cast<const float2*>(rope_table);
  if (dtype == CBK_BF16)
    rope_rows_kernel<CBK_BF16><<<grid_for(items, 256), 256, 0, st>>>(
        static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), n_rows, n_heads, head_dim,
        tab, table_rows, positions, rope_mode, status);
  else
    rope_rows_kernel<CBK_F16><<<grid_for(items, 256), 256, 0, st>>>(
        static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), n_rows, n_heads, head_dim,
        tab, table_rows, positions, rope_mode, status);
  return check_launch("rope_rows_kernel");
}

extern "C" int cbk_rope_scatter(const void* q_src, int64_t q_row_stride, const void* k_src,
                                int64_t k_row_stride, const void* v_src, int64_t v_row_stride,
                                int gather, const int64_t* idx, int64_t n_sel, int64_t S,
                                int n_q_heads, int n_kv_heads, int head_dim, int dtype,
                                const void* rope_table, int64_t table_rows, int rope_mode,
                                void* q_out, void* k_cache, void* v_cache, int32_t* status,
                                void* stream) {
  if (int rc = check_geometry("cbk_rope_scatter", n_kv_heads, head_dim, dtype)) return rc;
  if (int rc = check_mode("cbk_rope_scatter", rope_mode)) return rc;
  if (n_q_heads <= 0 || n_q_heads % n_kv_heads != 0)
    return set_error(CBK_ERR_INVALID, "cbk_rope_scatter: n_q_heads must be a multiple of n_kv_heads");
  if (!q_src || !k_src || !v_src || !idx || !rope_table || !q_out || !k_cache || !v_cache)
    return set_error(CBK_ERR_INVALID, "cbk_rope_scatter: null pointer argument");
  if (n_sel < 0 || S <= 0) return set_error(CBK_ERR_INVALID, "cbk_rope_scatter: bad sizes");
  if (!aligned16(q_src) || !aligned16(k_src) || !aligned16(v_src) || !aligned16(q_out) ||
      !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(rope_table) ||
      q_row_stride % 8 || k_row_stride % 8 || v_row_stride % 8)
    return set_error(CBK_ERR_INVALID,
                     "cbk_rope_scatter: buffers must be 16-byte aligned, row strides multiples of 8");
  if (n_sel == 0) return CBK_OK;
  const int gpr = head_dim >> 4;
  const int64_t items = n_sel * (n_q_heads * gpr + n_kv_heads * gpr + n_kv_heads * head_dim / 8);
  auto st = static_cast<cudaStream_t>(stream);
  auto tab = static_cast<const float2*>(rope_table);
#define CBK_LAUNCH_SCATTER(DT)                                                                  \
  rope_scatter_kernel<DT><<<grid_for(items, 256), 256, 0, st>>>(                                \
      static_cast<const uint16_t*>(q_src), q_row_stride, static_cast<const uint16_t*>(k_src),   \
      k_row_stride, static_cast<const uint16_t*>(v_src), v_row_stride, gather, idx, n_sel, S,   \
      n_q_heads, n_kv_heads, head_dim, tab, table_rows, rope_mode,                              \
      static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_cache),                          \
      static_cast<uint16_t*>(v_cache), status)
  if (dtype == CBK_BF16) CBK_LAUNCH_SCATTER(CBK_BF16); else CBK_LAUNCH_SCATTER(CBK_F16);
#undef CBK_LAUNCH_SCATTER
  return check_launch("rope_scatter_kernel");
}
