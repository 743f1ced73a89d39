// RoPE table, chunk-KV assembly (concat + RoPE shift), row RoPE and the
// per-layer fresh-row RoPE + scatter.  All of these are HBM-bound byte movers:
// 128-bit loads/stores, one pass over the data, rotation in registers (packed
// 16-bit ops for the torch-rounded mode, fp32 for the fp32 mode).
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
// It runs on packed 16-bit pairs (mul/add/sub.rn.{bf16x2,f16x2}): torch rounds
// the fp32 result of each op, and for 16-bit operands that fp32 result is the
// exact one wherever the rounding can tell (a product of two 8- or 11-bit
// significands fits fp32's 24; a sum whose operands' exponents differ by more
// than 24 - 8 bits lands within half an ulp of the larger operand either way),
// so one correctly rounded 16-bit op gives the same bits as torch's two steps
// (Pk in cbk_common.cuh).
// ---------------------------------------------------------------------------
// c4: the table entries (cos, sin) of 8 consecutive frequencies, as 4 float4
template <int DT>
__device__ __forceinline__ void rope8t(const uint4& lo, const uint4& hi, const float4 (&c4)[4],
                                       int mode, uint4& olo, uint4& ohi) {
  float2 t[8];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    t[2 * q] = make_float2(c4[q].x, c4[q].y);
    t[2 * q + 1] = make_float2(c4[q].z, c4[q].w);
  }
  if (mode == CBK_ROPE_REF) {
    const uint32_t* al = reinterpret_cast<const uint32_t*>(&lo);
    const uint32_t* bh = reinterpret_cast<const uint32_t*>(&hi);
    uint32_t* yl = reinterpret_cast<uint32_t*>(&olo);
    uint32_t* yh = reinterpret_cast<uint32_t*>(&ohi);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t c = Pk<DT>::cvt(t[2 * w].x, t[2 * w + 1].x);
      const uint32_t s = Pk<DT>::cvt(t[2 * w].y, t[2 * w + 1].y);
      yl[w] = Pk<DT>::sub(Pk<DT>::mul(al[w], c), Pk<DT>::mul(bh[w], s));
      yh[w] = Pk<DT>::add(Pk<DT>::mul(bh[w], c), Pk<DT>::mul(al[w], s));
    }
    return;
  }
  const uint16_t* xl = reinterpret_cast<const uint16_t*>(&lo);
  const uint16_t* xh = reinterpret_cast<const uint16_t*>(&hi);
  uint16_t* yl = reinterpret_cast<uint16_t*>(&olo);
  uint16_t* yh = reinterpret_cast<uint16_t*>(&ohi);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a = Elem<DT>::to_f(xl[e]);
    const float b = Elem<DT>::to_f(xh[e]);
    const float c = t[e].x, s = t[e].y;
    {
      yl[e] = Elem<DT>::from_f(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)));
      yh[e] = Elem<DT>::from_f(__fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s)));
    }
  }
}

template <int DT>
__device__ __forceinline__ void rope8(const uint4& lo, const uint4& hi, const float2* cs,
                                      int mode, uint4& olo, uint4& ohi) {
  const float4* p = reinterpret_cast<const float4*>(cs);
  const float4 c4[4] = {p[0], p[1], p[2], p[3]};
  rope8t<DT>(lo, hi, c4, mode, olo, ohi);
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
// (a)+(b) assemble: one layer per blockIdx.y, kAsmRows * kAsmRowIters rows per
// block, two warps per row set: the even warp rotates the rows' K (pair groups
// of 8 (lo, hi) elements), the odd warp copies their V (16-byte vectors).  A
// warp pass covers as many of its rows as fit 32 lanes x a batch (2 K groups =
// 4 vectors, or 4 V vectors per lane): one row of a 1024-wide K/V, four rows of
// a 128-wide one (a rank holding one KV head), so a warp keeps ~2 KB in flight
// whatever the row width.  Each lane issues all the loads of its batch before
// any arithmetic or store.
// ---------------------------------------------------------------------------
constexpr int kAsmThreads = 256;
constexpr int kAsmRows = kAsmThreads / 64;   // warp pairs per block
constexpr int kAsmRowIters = 4;               // rows per warp pair (rows it * kAsmRows + pair)
constexpr int kMaxChunksSmem = 2048;
constexpr int kAsmKBatch = 2;     // K pair groups per lane per batch
constexpr int kAsmVBatch = 4;     // V vectors per lane per batch

template <int DT>
__global__ void __launch_bounds__(kAsmThreads, 3)
assemble_kernel(const cbk_chunk_src* __restrict__ srcs, const int64_t* __restrict__ chunk_start,
                int n_chunks, int64_t S, int n_kv_heads, int head_dim,
                const float2* __restrict__ table, int64_t table_rows,
                const int64_t* __restrict__ positions, int mode, uint16_t* __restrict__ k_out,
                uint16_t* __restrict__ v_out, int64_t layer_stride, int32_t* status) {
  __shared__ int64_t s_start[kMaxChunksSmem + 1];
  const int layer = blockIdx.y;
  for (int c = threadIdx.x; c <= n_chunks; c += blockDim.x) s_start[c] = chunk_start[c];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_dim = n_kv_heads * head_dim;
  const int gph = head_dim >> 4;               // pair groups per head
  const int half = head_dim >> 1;
  const bool is_k = (warp & 1) == 0;
  const int per_row = is_k ? n_kv_heads * gph : kv_dim >> 3;          // K groups or V vectors
  const int slots = 32 * (is_k ? kAsmKBatch : kAsmVBatch);            // per lane batch x 32 lanes
  const int rpp = max(1, min(kAsmRowIters, slots / per_row));          // rows of this warp per pass
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kAsmRowIters * kAsmRows + (warp >> 1);
  // row it of this warp pair, its chunk and its row inside the chunk
  auto row_of = [&](int it, int64_t& t, int& c, int64_t& local) {
    t = row0 + static_cast<int64_t>(it) * kAsmRows;
    int lo = 0, hi = n_chunks - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_start[mid] <= t) lo = mid; else hi = mid - 1;
    }
    c = lo;
    local = t - s_start[lo];
  };
  if (rpp == 1) {
    // wide rows (a warp pass holds one row or less): one row at a time, its chunk,
    // position and source pointer warp-uniform
    for (int it = 0; it < kAsmRowIters; ++it) {
      int64_t t, local;
      int c;
      row_of(it, t, c, local);
      if (t >= S) break;
      const cbk_chunk_src src = srcs[static_cast<int64_t>(layer) * n_chunks + c];
      if (is_k) {
        const int64_t p = positions ? positions[t] : t;
        if (p < 0 || p >= table_rows) {
          if (lane == 0) report(status, CBK_STATUS_BAD_INDEX);
          continue;
        }
        const uint16_t* krow = static_cast<const uint16_t*>(src.k) + local * kv_dim;
        uint16_t* drow = k_out + layer * layer_stride + t * kv_dim;
        const float2* cs = table + p * half;
        for (int g0 = 0; g0 < per_row; g0 += 32 * kAsmKBatch) {
          uint4 xl[kAsmKBatch], xh[kAsmKBatch];
#pragma unroll
          for (int q = 0; q < kAsmKBatch; ++q) {
            const int g = g0 + q * 32 + lane;
            if (g < per_row) {
              const int off = (g / gph) * head_dim + (g % gph) * 8;
              xl[q] = ld_stream(krow + off);
              xh[q] = ld_stream(krow + off + half);
            }
          }
#pragma unroll
          for (int q = 0; q < kAsmKBatch; ++q) {
            const int g = g0 + q * 32 + lane;
            if (g < per_row) {
              const int off = (g / gph) * head_dim + (g % gph) * 8;
              uint4 ol, oh;
              rope8<DT>(xl[q], xh[q], cs + (g % gph) * 8, mode, ol, oh);
              st_vec(drow + off, ol);
              st_vec(drow + off + half, oh);
            }
          }
        }
      } else {
        const uint16_t* vrow = static_cast<const uint16_t*>(src.v) + local * kv_dim;
        uint16_t* drow = v_out + layer * layer_stride + t * kv_dim;
        for (int v0 = 0; v0 < per_row; v0 += 32 * kAsmVBatch) {
          uint4 x[kAsmVBatch];
#pragma unroll
          for (int q = 0; q < kAsmVBatch; ++q) {
            const int v = v0 + q * 32 + lane;
            if (v < per_row) x[q] = ld_stream(vrow + v * 8);
          }
#pragma unroll
          for (int q = 0; q < kAsmVBatch; ++q) {
            const int v = v0 + q * 32 + lane;
            if (v < per_row) st_vec(drow + v * 8, x[q]);
          }
        }
      }
    }
    return;
  }
  // narrow rows: rpp of this warp's rows per pass, each lane on its own (row, group)
  for (int it0 = 0; it0 < kAsmRowIters; it0 += rpp) {
    const int span = rpp * per_row;                                    // slots of this pass
    if (is_k) {
      for (int s0 = 0; s0 < span; s0 += 32 * kAsmKBatch) {
        // loads first, the rows' positions with them (addresses recomputed for the
        // stores: fewer live registers)
        uint4 xl[kAsmKBatch], xh[kAsmKBatch];
        int64_t pq[kAsmKBatch];
#pragma unroll
        for (int q = 0; q < kAsmKBatch; ++q) {
          const int sl = s0 + q * 32 + lane;
          const int it = it0 + sl / per_row, g = sl % per_row;
          if (sl >= span || it >= kAsmRowIters) continue;
          int64_t t, local;
          int c;
          row_of(it, t, c, local);
          if (t >= S) continue;
          pq[q] = positions ? positions[t] : t;
          const int off = (g / gph) * head_dim + (g % gph) * 8;
          const uint16_t* krow =
              static_cast<const uint16_t*>(srcs[static_cast<int64_t>(layer) * n_chunks + c].k) + local * kv_dim;
          xl[q] = ld_stream(krow + off);
          xh[q] = ld_stream(krow + off + half);
        }
#pragma unroll
        for (int q = 0; q < kAsmKBatch; ++q) {
          const int sl = s0 + q * 32 + lane;
          const int it = it0 + sl / per_row, g = sl % per_row;
          if (sl >= span || it >= kAsmRowIters) continue;
          const int64_t t = row0 + static_cast<int64_t>(it) * kAsmRows;
          if (t >= S) continue;
          const int64_t p = pq[q];
          if (p < 0 || p >= table_rows) {
            report(status, CBK_STATUS_BAD_INDEX);
            continue;
          }
          const int off = (g / gph) * head_dim + (g % gph) * 8;
          uint4 ol, oh;
          rope8<DT>(xl[q], xh[q], table + p * half + (g % gph) * 8, mode, ol, oh);
          uint16_t* d = k_out + layer * layer_stride + t * kv_dim + off;
          st_vec(d, ol);
          st_vec(d + half, oh);
        }
      }
    } else {
      for (int s0 = 0; s0 < span; s0 += 32 * kAsmVBatch) {
        uint4 x[kAsmVBatch];
#pragma unroll
        for (int q = 0; q < kAsmVBatch; ++q) {
          const int sl = s0 + q * 32 + lane;
          const int it = it0 + sl / per_row, v = sl % per_row;
          if (sl >= span || it >= kAsmRowIters) continue;
          int64_t t, local;
          int c;
          row_of(it, t, c, local);
          if (t >= S) continue;
          x[q] = ld_stream(static_cast<const uint16_t*>(srcs[static_cast<int64_t>(layer) * n_chunks + c].v) +
                           local * kv_dim + v * 8);
        }
#pragma unroll
        for (int q = 0; q < kAsmVBatch; ++q) {
          const int sl = s0 + q * 32 + lane;
          const int it = it0 + sl / per_row, v = sl % per_row;
          if (sl >= span || it >= kAsmRowIters) continue;
          const int64_t t = row0 + static_cast<int64_t>(it) * kAsmRows;
          if (t >= S) continue;
          st_vec(v_out + layer * layer_stride + t * kv_dim + v * 8, x[q]);
        }
      }
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
// fused cache at the selected positions.  Q, K and V rows are all read and
// written as 8-element (lo, hi) pair groups -- elements [8f, 8f+8) and
// [8f+D/2, 8f+D/2+8) of a head, f < D/16 -- rotated for Q and K, copied for V.
// A unit is 64 groups (2 KB, two groups per lane); a selected row has
// ceil(Hq*D/16 / 64) Q units, then ceil(Hkv*D/16 / 64) K units and as many V
// units.  A warp pass takes kScatUnits consecutive units of one row and issues
// every load of the pass -- the row's position, its source vectors, the
// cos/sin slice -- before the first rotation or store.  When D/16 divides 32,
// lane L always holds pair group L mod D/16 of some head: its element offset
// is the unit's first group * 16 + a per-lane constant, and one 8-entry
// cos/sin slice per lane serves every unit of the pass.
// ---------------------------------------------------------------------------
// Units per pass and CTAs per SM, measured at [32 layers, 3277 of 32768 rows,
// 32 Q / 8 KV heads, D = 128] with every source row read from HBM: 1 unit at
// 4 CTAs/SM (64 registers) 16.4 us per launch; 2 at 3 CTAs 17.4; 3 at 2 CTAs
// 17.0; 2 at 4 CTAs spills and takes 23 us.
constexpr int kScatGroups = 2;    // pair groups per lane per unit
#ifndef CBK_SCAT_UNITS
#define CBK_SCAT_UNITS 1
#endif
#ifndef CBK_SCAT_MINB
#define CBK_SCAT_MINB 4
#endif
constexpr int kScatUnits = CBK_SCAT_UNITS;

__device__ __forceinline__ void ld_cs(const float2* cs, float4 (&c4)[4]) {
  const float4* p = reinterpret_cast<const float4*>(cs);
#pragma unroll
  for (int q = 0; q < 4; ++q) c4[q] = p[q];
}

// GPR: pair groups per head (head_dim / 16) when fixed at compile time, else 0;
// MODE: the RoPE mode (a template parameter, so each instance holds one path)
template <int DT, int GPR, int MODE>
__global__ void __launch_bounds__(256, CBK_SCAT_MINB)
rope_scatter_kernel(const uint16_t* __restrict__ q_src, int64_t q_stride,
                    const uint16_t* __restrict__ k_src, int64_t k_stride,
                    const uint16_t* __restrict__ v_src, int64_t v_stride, int gather,
                    const int64_t* __restrict__ idx, int64_t n_sel, int64_t S, int n_q_heads,
                    int n_kv_heads, int head_dim, const float2* __restrict__ table,
                    int64_t table_rows, int by_row, uint16_t* __restrict__ q_out,
                    uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache,
                    int32_t* status) {
  constexpr int U = kScatUnits;
  constexpr int kUnitGroups = 32 * kScatGroups;
  const int lane = threadIdx.x & 31;
  if (GPR) head_dim = GPR * 16;
  const int gpr = head_dim >> 4;
  const int half = head_dim >> 1;
  const int qg = n_q_heads * gpr;
  const int kg = n_kv_heads * gpr;
  const int kv_dim = n_kv_heads * head_dim;
  const int64_t q_dim = static_cast<int64_t>(n_q_heads) * head_dim;
  const int nq = (qg + kUnitGroups - 1) / kUnitGroups;
  const int nk = (kg + kUnitGroups - 1) / kUnitGroups;
  const int per = nq + 2 * nk;
  const int passes = (per + U - 1) / U;         // warp passes per row
  const bool shared_f = (32 % gpr) == 0;
  const int lane_off = (lane / gpr) * head_dim + (lane % gpr) * 8;
  // element offset (lo half) of group `first + 32 q + lane`
  auto offset = [&](int first, int q) -> int {
    if (shared_f) return (first + 32 * q) * 16 + lane_off;
    const int g = first + 32 * q + lane;
    return (g / gpr) * head_dim + (g % gpr) * 8;
  };
  const int64_t n_items = n_sel * passes;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       w < n_items; w += warps) {
    const int64_t j = w / passes;
    const int part0 = static_cast<int>(w - j * passes) * U;
    int kind[U], first[U];   // kind: 0 Q, 1 K, 2 V, -1 past the row's end
    bool rope = false;
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int part = part0 + k;
      kind[k] = part >= per ? -1 : part < nq ? 0 : (part < nq + nk ? 1 : 2);
      first[k] = (part - (kind[k] == 0 ? 0 : kind[k] == 1 ? nq : nq + nk)) * kUnitGroups;
      rope |= kind[k] == 0 || kind[k] == 1;
    }
    uint4 x[U][2 * kScatGroups];
    auto load = [&](int64_t r) {
#pragma unroll
      for (int k = 0; k < U; ++k) {
        if (kind[k] < 0) continue;
        const uint16_t* src = kind[k] == 0 ? q_src + r * q_stride
                            : kind[k] == 1 ? k_src + r * k_stride : v_src + r * v_stride;
        const int ng = kind[k] == 0 ? qg : kg;
#pragma unroll
        for (int q = 0; q < kScatGroups; ++q) {
          if (first[k] + 32 * q + lane < ng) {
            const int o = offset(first[k], q);
            x[k][2 * q] = ld_vec(src + o);
            x[k][2 * q + 1] = ld_vec(src + o + half);
          }
        }
      }
    };
    const int64_t p = idx[j];
    // without a gather the source row is j: its loads go out before the position
    // arrives, and with a table indexed by row (row j holds the cos/sin of idx[j])
    // so do the cos/sin loads -- the whole pass waits for memory once
    if (!gather) load(j);
    float4 c4[4];
    if (by_row && rope && shared_f && j < table_rows) ld_cs(table + j * half + (lane % gpr) * 8, c4);
    if (p < 0 || p >= S || (by_row ? j >= table_rows : p >= table_rows)) {
      if (lane == 0) report(status, CBK_STATUS_BAD_INDEX);
      continue;
    }
    if (gather) load(p);
    const float2* cs = table + (by_row ? j : p) * half;
    if (!by_row && rope && shared_f) ld_cs(cs + (lane % gpr) * 8, c4);
#pragma unroll
    for (int k = 0; k < U; ++k) {
      if (kind[k] < 0) continue;
      uint16_t* dst = kind[k] == 0 ? q_out + j * q_dim : (kind[k] == 1 ? k_cache : v_cache) + p * kv_dim;
      const int ng = kind[k] == 0 ? qg : kg;
#pragma unroll
      for (int q = 0; q < kScatGroups; ++q) {
        const int g = first[k] + 32 * q + lane;
        if (g < ng) {
          const int o = offset(first[k], q);
          uint4 lo = x[k][2 * q], hi = x[k][2 * q + 1];
          if (kind[k] != 2) {
            if (!shared_f) ld_cs(cs + (g % gpr) * 8, c4);
            const uint4 a = lo, b = hi;
            rope8t<DT>(a, b, c4, MODE, lo, hi);
          }
          st_vec(dst + o, lo);
          st_vec(dst + o + half, hi);
        }
      }
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
  const int64_t rows_per_block = static_cast<int64_t>(kAsmRows) * kAsmRowIters;
  dim3 grid(static_cast<unsigned>((S + rows_per_block - 1) / rows_per_block), static_cast<unsigned>(n_layers));
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
  const int by_row = (rope_mode & CBK_ROPE_TABLE_BY_ROW) ? 1 : 0;
  rope_mode &= ~CBK_ROPE_TABLE_BY_ROW;
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
  const int64_t per = (n_q_heads * gpr + 32 * kScatGroups - 1) / (32 * kScatGroups) +
                      2 * ((n_kv_heads * gpr + 32 * kScatGroups - 1) / (32 * kScatGroups));
  const int64_t warp_items = n_sel * ((per + kScatUnits - 1) / kScatUnits);   // 8 warps per block
  auto st = static_cast<cudaStream_t>(stream);
  auto tab = static_cast<const float2*>(rope_table);
#define CBK_LAUNCH_SCATTER(DT, GPR, MODE)                                                       \
  rope_scatter_kernel<DT, GPR, MODE><<<grid_for(warp_items * 32, 256, 148 * 64), 256, 0, st>>>(   \
      static_cast<const uint16_t*>(q_src), q_row_stride, static_cast<const uint16_t*>(k_src),   \
      k_row_stride, static_cast<const uint16_t*>(v_src), v_row_stride, gather, idx, n_sel, S,   \
      n_q_heads, n_kv_heads, head_dim, tab, table_rows, by_row,                                 \
      static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_cache),                          \
      static_cast<uint16_t*>(v_cache), status)
#define CBK_LAUNCH_SCATTER_M(DT, GPR)                                                           \
  if (rope_mode == CBK_ROPE_REF) CBK_LAUNCH_SCATTER(DT, GPR, CBK_ROPE_REF);                     \
  else CBK_LAUNCH_SCATTER(DT, GPR, CBK_ROPE_FP32)
#define CBK_LAUNCH_SCATTER_DT(GPR)                                                              \
  if (dtype == CBK_BF16) { CBK_LAUNCH_SCATTER_M(CBK_BF16, GPR); } else { CBK_LAUNCH_SCATTER_M(CBK_F16, GPR); }
  if (head_dim == 128) {
    CBK_LAUNCH_SCATTER_DT(8);
  } else {
    CBK_LAUNCH_SCATTER_DT(0);
  }
#undef CBK_LAUNCH_SCATTER_DT
#undef CBK_LAUNCH_SCATTER_M
#undef CBK_LAUNCH_SCATTER
  return check_launch("rope_scatter_kernel");
}
