// Partial-query attention on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Work item = (KV head, pair of 128-row Q tiles, range of key tiles).  Rows of a
// tile are r = tok * G + h (G = q heads per KV head, 128 / G selected tokens per
// tile), so K/V tiles are shared by the GQA group without expanding them.  Keys
// are visited in 128-key tiles; causality is a per-row position compare (no
// mask tensor): on a diagonal key tile the invisible scores are set to -inf in
// registers, and the tile then runs the same code as a fully visible one.
//
// Work plan (attn_plan_kernel, on the device from the positions, so no host
// synchronisation; reusable by every layer that attends with the same
// positions): the (KV head, pair, key tile) steps of the call are laid end to
// end and cut into one equal range per SM ("worker"); a pair whose steps cross
// a cut is split into pieces, whose partial results attn_combine_kernel
// merges.  Every SM gets the same number of steps, whatever the spread of the
// pairs' key ranges (a causal selection makes them range from one tile to all).
//
// The attention kernel is persistent: one CTA per SM keeps its TMEM and
// barriers; CTA b runs worker b, then takes further workers from a queue in the
// workspace (none are left when every CTA is resident), running the items of a
// worker in order.  The producer
// publishes each item to the other warps through a two-slot ring in shared
// memory and loads the next item's Q as soon as the current item's last
// S = Q K^T has been issued, so set-up costs overlap the previous item.  The
// copies go out in the order the first MMAs need them (Q tile 0, K, Q tile 1,
// V), and the first worker needs no queue round trip, which shortens the
// start of the call, when every CTA loads at once.
//
// TMEM (512 columns): tile t uses S/P at [256t, 256t+128) and O at
// [256t+128, 256t+128+D).  S lands in fp32; the softmax warps write P back in
// place as packed 16-bit pairs and the PV MMA reads P straight from TMEM (A
// operand in tensor memory), so P never touches shared memory.
//
// Warp roles (384 threads):
//   warp 0        producer: fetches items, loads both Q tiles, then K and V tiles
//                 into two separate 2-stage rings (TMA; one elected lane issues)
//   warp 1        MMA issuer (one elected lane of the converged warp): per key
//                 tile j, for t = 0, 1: O_t += P_t(j) V(j) over keys 0-63 as
//                 soon as the softmax has stored that half of P, over keys
//                 64-127 once all of P is stored, then S_t(j+1) = Q_t K(j+1)^T.
//                 MMAs issued by one lane run in order, so S_t(j+1) overwrites
//                 P_t(j) only after the PV that reads it; while one tile's
//                 softmax runs, the tensor core works on the other tile.
//   warp 2        TMEM allocator
//   warps 4..7    softmax of tile 0; warps 8..11 softmax of tile 1.  Thread i of
//                 warp w owns TMEM lane 32*(w%4)+i, i.e. one row: max / exp / sum
//                 are thread-local.  O is rescaled only when the running max
//                 grows by more than 2^8 (O / l uses the same stale max).
// Barrier phases are counted across items.  Every mbarrier wait is bounded
// (2 s of wall time); on timeout the kernel sets CBK_STATUS_TIMEOUT, drains its
// own TMA copies and MMAs, frees TMEM and returns.
#include <algorithm>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "cbk_common.cuh"

namespace cbk {

constexpr int kBM = 128;       // rows per Q tile
constexpr int kBN = 128;       // keys per KV tile
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxKvTiles = 2049;          // S <= 262144

// Fixed cost of one work item in key-tile steps (Q load, pipeline refill and
// epilogue of a Q-tile pair), for the plan's balance.
#ifndef CBK_ATTN_ITEM_COST
#define CBK_ATTN_ITEM_COST 2
#endif
constexpr int kAttnItemCost = CBK_ATTN_ITEM_COST;
#ifndef CBK_ATTN_WORKERS_PER_SM
#define CBK_ATTN_WORKERS_PER_SM 1
#endif
constexpr int kAttnWorkersPerSm = CBK_ATTN_WORKERS_PER_SM;
// Share of the cost (percent) left to a dynamic tail of whole short units.
#ifndef CBK_ATTN_DYN_PCT
#define CBK_ATTN_DYN_PCT 0
#endif
constexpr int kAttnDynPct = CBK_ATTN_DYN_PCT;
// PV of a key tile in two halves: the softmax warps release the first 64 keys'
// P once it is stored, so PV over them runs while the last 64 are exponentiated,
// and the next S = QK^T (which overwrites P) follows the second half sooner.
#ifndef CBK_ATTN_PV_SPLIT
#define CBK_ATTN_PV_SPLIT 1
#endif
constexpr bool kPvSplit = CBK_ATTN_PV_SPLIT != 0;

template <int HD>
struct AttnSmem {
  static constexpr int kQBytes = kBM * HD * 2;     // one Q tile
  static constexpr int kKVBytes = kBN * HD * 2;    // one K or V tile
  static constexpr int kQ = 0;                     // 2 Q tiles
  static constexpr int kK0 = kQ + 2 * kQBytes;     // 2 K stages
  static constexpr int kV0 = kK0 + 2 * kKVBytes;   // 2 V stages
  static constexpr int kBar = kV0 + 2 * kKVBytes;  // 32 x 8-byte barriers
  static constexpr int kItems = kBar + 32 * 8;     // 2-slot item ring (int4)
  static constexpr int kMisc = kItems + 2 * 16;    // tmem slot + abort flag
  static constexpr int kTotal = kMisc + 16;
  // at least 120 KB so that one CTA (holding all 512 TMEM columns) fills an SM
  static constexpr int kAlloc = (kTotal + 1024) > 122880 ? (kTotal + 1024) : 122880;
};

enum Bar { B_QFULL = 0, B_QEMPTY = 1, B_KFULL = 2, B_KEMPTY = 4, B_VFULL = 6, B_VEMPTY = 8,
           B_SFULL = 10, B_PFULL = 12, B_ODONE = 14, B_OFREE = 16, B_IFULL = 18, B_IEMPTY = 20,
           B_DRAIN = 22, B_QFULL1 = 23, B_PHALF = 24 };
// B_QFULL: Q tile 0 landed, B_QFULL1: Q tile 1; B_PHALF + t: the first half of
// tile t's P (keys 0-63 of the key tile) is in TMEM

// Work plan in the caller's workspace (written by attn_plan_kernel).
struct AttnPlanHeader {
  int n_items;     // work items
  int n_workers;   // equal ranges of steps (one per SM)
  int n_slots;     // partial-result slots in use
  int error;       // nonzero: the plan did not fit the workspace bounds
  int next_item;   // worker queue head: zeroed by the plan and after every attention call
  int n_split;     // Q tiles (over all KV heads) whose key range is split
};

struct AttnParams {
  const int64_t* pos;
  uint16_t* out;
  int32_t* status;
  const AttnPlanHeader* plan;
  int* queue;             // &plan->next_item
  const int4* items;      // (kv head, tile pair, first key tile j0, j1 | piece << 16) by worker
  const int* first_item;  // [n_workers + 1]: the items of worker w are [first_item[w], first_item[w+1])
  const int* tile_base;   // [Hkv][n_tiles]: first partial slot of a split tile, -1 if not split
  const int4* split_desc; // [n_split]: (kvh * n_tiles + tile, first slot, chunks, 0) per split tile
  uint16_t* part_o;       // [slot][128][HD] O / l of the chunk, in the inputs' 16-bit type
                          // (a convex combination of V rows: bounded by max |V|, so it
                          // cannot overflow the type V itself is stored in)
  float2* part_ml;        // [slot][128] (running max in log2 units, row sum)
  int64_t n_sel;
  int n_q_heads;
  int group;          // G
  int tok_per_tile;   // 128 / G
  int n_tiles;        // Q tiles per KV head
  float scale_log2;
  int store_v8;       // out and workspace are 32-byte aligned: 32-byte epilogue stores
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

// two fp32 -> one packed 16-bit pair (lo in the low half), one conversion instruction
template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (DT == CBK_BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

// 32 fp32 values of a row times inv, rounded to the 16-bit type, stored to dst: as
// two 32-byte stores (whole sectors) when the caller's buffers are 32-byte aligned,
// else as four 16-byte stores.  The epilogue's stores are scattered rows (one row
// per thread), so whole-sector stores halve the requests and leave no partial sector.
template <int DT>
__device__ __forceinline__ void store_chunk(uint16_t* dst, const uint32_t (&o)[32], float inv, bool v8) {
  uint32_t w[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) w[e] = pack2<DT>(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
  if (v8) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
      asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                   :: "l"(dst + 16 * h), "r"(w[8 * h]), "r"(w[8 * h + 1]), "r"(w[8 * h + 2]), "r"(w[8 * h + 3]),
                      "r"(w[8 * h + 4]), "r"(w[8 * h + 5]), "r"(w[8 * h + 6]), "r"(w[8 * h + 7])
                   : "memory");
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) st_vec(dst + 8 * q, make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]));
  }
}

// max of three (one instruction on sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

// (d0, d1) = (a0, a1) * (b, b) + (c, c) as one packed fp32 pair instruction
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\tmov.b64 rc, {%5, %5};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b), "f"(c));
}

// (d0, d1) += (a0, a1) as one packed fp32 pair instruction
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1) {
  asm("{\n\t.reg .b64 ra, rd;\n\t"
      "mov.b64 rd, {%0, %1};\n\tmov.b64 ra, {%2, %3};\n\t"
      "add.f32x2 rd, rd, ra;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d0), "+f"(d1) : "f"(a0), "f"(a1));
}

// packed fp32 pairs (two floats in one 64-bit register pair) for the f32x2 instructions
__device__ __forceinline__ uint64_t pk_f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk_f2(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for a pair on the FMA pipe, to take load off the exponential unit.
// Split x = j + f with j = rint(x) (adding 1.5 * 2^23 leaves rint(x) in the low
// mantissa bits) and f in [-0.5, 0.5]; 2^f by a degree-3 polynomial, the
// minimax fit for relative error on [-0.5, 0.5] found with the Remez exchange
// algorithm (max relative error 7.5e-5, below the 16-bit rounding of P); 2^j is
// added into the exponent field.  x is clamped at -126 (j >= -126 keeps the
// exponent field from borrowing into the sign); below that the result is a
// denormal ~1e-38 instead of 0.
__device__ __forceinline__ void exp2_fma_pair(float x0, float x1, float& y0, float& y1) {
  constexpr float kMagic = 12582912.f;   // 1.5 * 2^23
  const uint64_t X = pk_f2(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t M = pk_f2(kMagic, kMagic);
  const uint64_t T = add_f2(X, M);
  const uint64_t F = sub_f2(X, sub_f2(T, M));
  uint64_t P = fma_f2(F, pk_f2(0.0551716685295105f, 0.0551716685295105f),
                      pk_f2(0.2426111251115799f, 0.2426111251115799f));
  P = fma_f2(P, F, pk_f2(0.6932609677314758f, 0.6932609677314758f));
  P = fma_f2(P, F, pk_f2(0.9999280571937561f, 0.9999280571937561f));
  float p0, p1, t0, t1;
  upk_f2(P, p0, p1);
  upk_f2(T, t0, t1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Pairs e (of the 16 per 32 columns; 3 of 16, the best of a 12-50 % sweep with PV
// split in halves and diagonal tiles masked in place; 6 of 16 was best before
// those) whose exponentials go to the FMA pipe; the others use ex2.approx.
#ifndef CBK_ATTN_EMU_MASK
#define CBK_ATTN_EMU_MASK 0x0421
#endif

// P = 2^(s * sl2 - m) of columns [32 c4, 32 c4 + 32) of a row, packed into 16-bit
// pairs, with the row sum accumulated in packed fp32 pairs.  3 of the 16 pairs go
// to the FMA-pipe polynomial.  Invisible keys arrive as s = -inf: ex2.approx gives
// 0 for them, the polynomial (its argument clamped at -126) 2^-126.
template <int DT>
__device__ __forceinline__ void exp_chunk(const uint32_t (&s)[kBN], int c4, float sl2, float neg_m,
                                          float& ra0, float& ra1, float& rb0, float& rb1, uint32_t (&pk)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int c = c4 * 32 + 2 * e;
    float x0, x1, p0, p1;
    fma2(x0, x1, __uint_as_float(s[c]), __uint_as_float(s[c + 1]), sl2, neg_m);
    if ((CBK_ATTN_EMU_MASK >> e) & 1) {
      exp2_fma_pair(x0, x1, p0, p1);
    } else {
      p0 = ex2(x0);
      p1 = ex2(x1);
    }
    if (e & 1) add2(rb0, rb1, p0, p1);
    else add2(ra0, ra1, p0, p1);
    pk[e] = pack2<DT>(p0, p1);
  }
}

// Pair p holds tiles 2p - o and 2p + 1 - o, o = n_tiles mod 2: with an odd
// count the tile without a partner is tile 0, the shortest, not the last one.
__device__ __forceinline__ int pair_tile(int n_tiles, int pair, int t) {
  return 2 * pair + t - (n_tiles & 1);
}

// Q tiles are aligned to the end of the selection: tile t holds tokens
// [n_sel - (n_tiles - t) * tok_per_tile, + tok_per_tile), so the one partly
// filled tile is tile 0, whose tokens come first and see the fewest keys (the
// last selected tokens, which see every key, fill whole tiles).  Tile 0's
// first token may be negative: those rows load as zeros and are not stored.
__device__ __forceinline__ int64_t tile_tok0(int64_t n_sel, int n_tiles, int tok_per_tile, int tile) {
  return n_sel - static_cast<int64_t>(n_tiles - tile) * tok_per_tile;
}

// number of 128-key tiles a Q tile needs (its last token has the largest position)
__device__ __forceinline__ int tile_key_tiles(const int64_t* pos, int64_t n_sel, int n_tiles, int tok_per_tile,
                                              int tile) {
  const int64_t last = tile_tok0(n_sel, n_tiles, tok_per_tile, tile) + tok_per_tile - 1;
  return static_cast<int>(pos[last] / kBN) + 1;
}

// geometry of one work item: Q-tile pair, range [j0, j1) of its key tiles
struct ItemGeom {
  int kvh, pair, piece, j0;
  int n_kv[2];          // key tiles of this item for tile 0 / 1 (0: tile absent or done)
  int n_all;            // max of the two
  int tile[2];           // tile index of slot 0 / 1 (out of range: slot empty)
  bool has[2];           // the slot holds a tile
  int64_t tok0[2], tok_end[2], p_max[2];
};

__device__ __forceinline__ ItemGeom item_geom(const int4 item, const AttnParams& prm) {
  ItemGeom g;
  g.kvh = item.x;
  g.pair = item.y;
  g.j0 = item.z;
  const int j1 = item.w & 0xFFFF;
  g.piece = item.w >> 16;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int tile = pair_tile(prm.n_tiles, g.pair, t);
    g.tile[t] = tile;
    g.has[t] = tile >= 0 && tile < prm.n_tiles;
    g.tok0[t] = tile_tok0(prm.n_sel, prm.n_tiles, prm.tok_per_tile, tile);
    if (!g.has[t]) {
      g.tok_end[t] = g.tok0[t];
      g.p_max[t] = 0;
      g.n_kv[t] = 0;
    } else {
      g.tok_end[t] = g.tok0[t] + prm.tok_per_tile;
      g.p_max[t] = prm.pos[g.tok_end[t] - 1];
      const int n_full = static_cast<int>(g.p_max[t] / kBN) + 1;
      g.n_kv[t] = max(0, min(j1, n_full) - g.j0);
    }
  }
  g.n_all = max(g.n_kv[0], g.n_kv[1]);
  return g;
}

template <int DT, int HD>
__global__ void __launch_bounds__(kThreads, 1)
partial_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const AttnParams prm) {
  using L = AttnSmem<HD>;
  if (prm.plan->error || prm.plan->n_items == 0) return;
  const int n_workers = prm.plan->n_workers;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - raw_addr);
  const uint32_t sQ = base + L::kQ, sK0 = base + L::kK0, sV0 = base + L::kV0;
  auto bar = [&](int i) { return base + L::kBar + 8u * i; };
  volatile int4* s_item = reinterpret_cast<volatile int4*>(sbase + L::kItems);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sbase + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sbase + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar(B_QFULL), 1);
    mbar_init(bar(B_QFULL1), 1);
    mbar_init(bar(B_QEMPTY), 1);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_KFULL + i), 1);
      mbar_init(bar(B_KEMPTY + i), 1);
      mbar_init(bar(B_VFULL + i), 1);
      mbar_init(bar(B_VEMPTY + i), 1);
      mbar_init(bar(B_SFULL + i), 1);
      mbar_init(bar(B_PFULL + i), 4);     // one arrive per softmax warp of the tile
      mbar_init(bar(B_PHALF + i), 4);
      mbar_init(bar(B_ODONE + i), 1);
      mbar_init(bar(B_OFREE + i), 4);
      mbar_init(bar(B_IFULL + i), 1);
      mbar_init(bar(B_IEMPTY + i), 9);    // MMA thread + 8 softmax warps
    }
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
  bool failed = false;

  // consumers: item n of this CTA from ring slot n & 1
  auto take_item = [&](int n, int4& item) -> bool {
    if (!wait_or_abort(bar(B_IFULL + (n & 1)), (n >> 1) & 1, abort_flag)) return false;
    const volatile int4& v = s_item[n & 1];
    item = make_int4(v.x, v.y, v.z, v.w);
    return true;
  };

  // warp-uniform bounded wait
  auto wait_all = [&](uint32_t b, uint32_t parity) {
    return __all_sync(0xffffffffu, wait_or_abort(b, parity, abort_flag));
  };

  if (warp == 0) {
    // ------------------------------------------------ item queue + TMA producer
    // The whole warp runs the loop; one elected lane issues (see elect_one).
    const bool leader = elect_one();
    const int leader_lane = __ffs(__ballot_sync(0xffffffffu, leader)) - 1;
    if (leader) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    int g = 0;                               // K/V tiles loaded by this CTA
    int last_k[2] = {-1, -1}, last_v[2] = {-1, -1};
    int n_q = 0;                             // Q loads issued
    int it = 0, it_end = 0;                  // items left of the current worker
    bool first_worker = true;
    for (int n = 0; !failed; ++n) {
      if (n >= 2 && !wait_all(bar(B_IEMPTY + (n & 1)), ((n >> 1) - 1) & 1)) {
        failed = true;
        break;
      }
      while (it >= it_end) {                 // next worker with items
        // worker b is CTA b's first (no round trip to the queue before the first
        // copies); the queue hands out workers gridDim.x, gridDim.x + 1, ...
        int w = blockIdx.x;
        if (!first_worker) {
          if (leader) w = static_cast<int>(gridDim.x) + atomicAdd(prm.queue, 1);
          w = __shfl_sync(0xffffffffu, w, leader_lane);
        }
        first_worker = false;
        if (w >= n_workers) {
          // no work left to hand out: the merge kernel (a programmatic dependent of
          // this one) may be scheduled as SMs free up; it waits for this grid to finish
          asm volatile("griddepcontrol.launch_dependents;");
          it = it_end = 0;
          break;
        }
        it = prm.first_item[w];
        it_end = prm.first_item[w + 1];
      }
      const int4 item = it < it_end ? prm.items[it++] : make_int4(-1, 0, 0, 0);
      if (leader) {
        s_item[n & 1].x = item.x;
        s_item[n & 1].y = item.y;
        s_item[n & 1].z = item.z;
        s_item[n & 1].w = item.w;
        mbar_arrive(bar(B_IFULL + (n & 1)));   // release: the slot is visible to the waiters
      }
      if (item.x < 0) break;
      // The copies need only the item's head, tiles and first key tile; the key-tile
      // count needs the positions, so it is read once the first copies are in flight.
      const int kvh = item.x, j0 = item.z;
      bool has[2];
      int tok0[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int tile = pair_tile(prm.n_tiles, item.y, t);
        has[t] = tile >= 0 && tile < prm.n_tiles;
        tok0[t] = static_cast<int>(tile_tok0(prm.n_sel, prm.n_tiles, prm.tok_per_tile, tile));
      }
      // Q of this item once the previous item's last S = Q K^T has been issued
      if (n_q > 0 && !wait_all(bar(B_QEMPTY), (n_q - 1) & 1)) {
        failed = true;
        break;
      }
      // Copies in the order the first MMAs need them: Q tile 0, K, Q tile 1, V (a
      // missing tile's barrier completes on the arrive alone)
      auto load_q = [&](int t) {
        if (!leader) return;
        const uint32_t b = bar(t ? B_QFULL1 : B_QFULL);
        mbar_expect_tx(b, has[t] ? L::kQBytes : 0);
        if (!has[t]) return;
#pragma unroll
        for (int h = 0; h < HD / 64; ++h)
          tma_load_3d(sQ + t * L::kQBytes + h * (kBM * 128), &tm_q, b, h * 64, kvh * prm.group, tok0[t]);
      };
      load_q(0);
      ++n_q;
      int n_all = 1;        // every item holds at least one key tile of its later Q tile
      for (int j = 0; j < n_all; ++j, ++g) {
        const int st = g & 1;
        if (g >= 2 && !wait_all(bar(B_KEMPTY + st), ((g >> 1) - 1) & 1)) {
          failed = true;
          break;
        }
        if (leader) {
          mbar_expect_tx(bar(B_KFULL + st), L::kKVBytes);
#pragma unroll
          for (int h = 0; h < HD / 64; ++h)
            tma_load_3d(sK0 + st * L::kKVBytes + h * (kBN * 128), &tm_k, bar(B_KFULL + st), h * 64, kvh,
                        (j0 + j) * kBN);
        }
        last_k[st] = g;
        if (j == 0) load_q(1);
        if (g >= 2 && !wait_all(bar(B_VEMPTY + st), ((g >> 1) - 1) & 1)) {
          failed = true;
          break;
        }
        if (leader) {
          mbar_expect_tx(bar(B_VFULL + st), L::kKVBytes);
#pragma unroll
          for (int h = 0; h < HD / 64; ++h)
            tma_load_3d(sV0 + st * L::kKVBytes + h * (kBN * 128), &tm_v, bar(B_VFULL + st), h * 64, kvh,
                        (j0 + j) * kBN);
        }
        last_v[st] = g;
        if (j == 0) n_all = item_geom(item, prm).n_all;
      }
    }
    // Drain: every armed copy must land before the CTA can retire.
    if (n_q > 0 && !__all_sync(0xffffffffu, mbar_wait(bar(B_QFULL), (n_q - 1) & 1))) failed = true;
    if (n_q > 0 && !__all_sync(0xffffffffu, mbar_wait(bar(B_QFULL1), (n_q - 1) & 1))) failed = true;
    for (int st = 0; st < 2; ++st) {
      if (last_k[st] >= 0 && !__all_sync(0xffffffffu, mbar_wait(bar(B_KFULL + st), (last_k[st] >> 1) & 1)))
        failed = true;
      if (last_v[st] >= 0 && !__all_sync(0xffffffffu, mbar_wait(bar(B_VFULL + st), (last_v[st] >> 1) & 1)))
        failed = true;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop; one elected lane issues the MMAs and commits
    // (see elect_one).
    const bool leader = elect_one();
    const uint32_t idesc_s = umma_idesc_f16(DT, kBM, kBN, 0);
    const uint32_t idesc_o = umma_idesc_f16(DT, kBM, HD, 1);
    // Base descriptors of the Q tiles and K/V stages, built once: a slice's
    // descriptor is its base plus the slice offset in 16-byte units (the start
    // address field; shared-memory offsets stay below 2^18 bytes, so no carry).
    uint64_t dq[2], dk[2], dv[2];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      dq[b] = umma_desc_sw128(sQ + b * L::kQBytes, 16, 1024);
      dk[b] = umma_desc_sw128(sK0 + b * L::kKVBytes, 16, 1024);
      dv[b] = umma_desc_sw128(sV0 + b * L::kKVBytes, kBN * 128, 1024);
    }
    auto issue_s = [&](int t, int g) {
      const uint64_t q0 = t ? dq[1] : dq[0];
      const uint64_t k0 = (g & 1) ? dk[1] : dk[0];
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint32_t off = ((kk >> 2) * (kBM * 128) + (kk & 3) * 32) >> 4;
        const uint32_t offk = ((kk >> 2) * (kBN * 128) + (kk & 3) * 32) >> 4;
        if (leader) umma_f16_ss(tmem + 256 * t, q0 + off, k0 + offk, idesc_s, kk > 0 ? 1u : 0u);
      }
      if (leader) umma_commit(bar(B_SFULL + t));
    };
    // O (+)= P V over the keys [16 kk_lo, 16 kk_hi) of the key tile
    auto issue_pv = [&](int t, int g, bool acc, int kk_lo, int kk_hi) {
      const uint64_t v0 = (g & 1) ? dv[1] : dv[0];
#pragma unroll
      for (int kk = kk_lo; kk < kk_hi; ++kk)
        if (leader)
          umma_f16_ts(tmem + 256 * t + kBN, tmem + 256 * t + kk * 8, v0 + ((kk * 16 * 128) >> 4), idesc_o,
                      (acc || kk > 0) ? 1u : 0u);
    };
    int g = 0;                 // K/V tiles consumed
    int pc[2] = {0, 0};        // P tiles consumed per Q-tile slot
    int oc[2] = {0, 0};        // O results handed to the epilogue per Q-tile slot
    for (int n = 0; !failed; ++n) {
      int4 item;
      if (!__all_sync(0xffffffffu, take_item(n, item))) {
        failed = true;
        break;
      }
      if (leader) mbar_arrive(bar(B_IEMPTY + (n & 1)));
      if (item.x < 0) break;
      const ItemGeom ig = item_geom(item, prm);
      if (!wait_all(bar(B_QFULL), n & 1) || !wait_all(bar(B_KFULL + (g & 1)), (g >> 1) & 1)) {
        failed = true;
        break;
      }
      tc_fence_after();
      // S(0): the previous item's PVs that read P from these columns were issued
      // earlier by this warp, so they complete first
      if (ig.n_kv[0] > 0) issue_s(0, g);
      if (!wait_all(bar(B_QFULL1), n & 1)) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (ig.n_kv[1] > 0) issue_s(1, g);
      if (leader) {
        umma_commit(bar(B_KEMPTY + (g & 1)));
        if (ig.n_all == 1) umma_commit(bar(B_QEMPTY));
      }
      for (int j = 0; j < ig.n_all && !failed; ++j) {
        const int gj = g + j;
        const bool next_k = j + 1 < ig.n_all;
        if (next_k && !wait_all(bar(B_KFULL + ((gj + 1) & 1)), ((gj + 1) >> 1) & 1)) {
          failed = true;
          break;
        }
        if (!wait_all(bar(B_VFULL + (gj & 1)), (gj >> 1) & 1)) {
          failed = true;
          break;
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int n_t = ig.n_kv[t];
          if (j >= n_t) continue;
          if (kPvSplit) {
            if (!wait_all(bar(B_PHALF + t), pc[t] & 1)) {
              failed = true;
              break;
            }
          } else if (!wait_all(bar(B_PFULL + t), pc[t] & 1)) {
            failed = true;
            break;
          }
          // the first PV of an item overwrites O: the previous epilogue must have read it
          if (j == 0 && oc[t] > 0 && !wait_all(bar(B_OFREE + t), (oc[t] - 1) & 1)) {
            failed = true;
            break;
          }
          tc_fence_after();
          if (kPvSplit) {
            issue_pv(t, gj, j > 0, 0, kBN / 32);
            if (!wait_all(bar(B_PFULL + t), pc[t] & 1)) {
              failed = true;
              break;
            }
            tc_fence_after();
            issue_pv(t, gj, true, kBN / 32, kBN / 16);
          } else {
            issue_pv(t, gj, j > 0, 0, kBN / 16);
          }
          ++pc[t];
          if (j + 1 < n_t) {
            issue_s(t, gj + 1);
          } else {
            if (leader) umma_commit(bar(B_ODONE + t));
            ++oc[t];
          }
        }
        if (failed) break;
        if (leader) {
          umma_commit(bar(B_VEMPTY + (gj & 1)));
          if (next_k) umma_commit(bar(B_KEMPTY + ((gj + 1) & 1)));
          if (j + 2 == ig.n_all) umma_commit(bar(B_QEMPTY));   // last S of the item issued
        }
      }
      g += ig.n_all;
    }
    // Drain: all MMAs issued by this warp complete before TMEM is released.
    if (leader) umma_commit(bar(B_DRAIN));
    if (!__all_sync(0xffffffffu, mbar_wait(bar(B_DRAIN), 0))) failed = true;
  } else if (warp >= 4) {
    // ----------------------------------------------- softmax + epilogue warps
    const int t = (warp - 4) >> 2;            // Q tile of this warpgroup
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const uint32_t tS = tmem + 256 * t + lane_off, tO = tS + kBN;
    const float sl2 = prm.scale_log2;
    int sc = 0;     // S tiles consumed
    int oc = 0;     // O results consumed
    for (int n = 0; !failed; ++n) {
      int4 item;
      if (!__all_sync(0xffffffffu, take_item(n, item))) {
        failed = true;
        break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_IEMPTY + (n & 1)));
      if (item.x < 0) break;
      const ItemGeom ig = item_geom(item, prm);
      // (t is warp-uniform; selects keep the geometry in registers)
      const int n_t = t ? ig.n_kv[1] : ig.n_kv[0];
      if (n_t == 0) continue;
      const int64_t tok = (t ? ig.tok0[1] : ig.tok0[0]) + row / prm.group;
      const bool row_valid = tok >= 0 && tok < (t ? ig.tok_end[1] : ig.tok_end[0]);
      const int64_t p_row = row_valid ? prm.pos[tok] : (t ? ig.p_max[1] : ig.p_max[0]);
      // first partial slot of the tile if its key range is split (read now, used by the epilogue)
      const int slot0 = prm.tile_base[ig.kvh * prm.n_tiles + (t ? ig.tile[1] : ig.tile[0])];
      float m_used = -INFINITY, l_sum = 0.f;
      for (int j = 0; j < n_t; ++j, ++sc) {
        if (!__all_sync(0xffffffffu, wait_or_abort(bar(B_SFULL + t), sc & 1, abort_flag))) {
          failed = true;
          break;
        }
        tc_fence_after();
        // keys (j0 + j)*kBN + c are visible to this row iff c <= lim
        const int64_t lim64 = p_row - static_cast<int64_t>(ig.j0 + j) * kBN;
        const int lim = lim64 >= kBN ? kBN : static_cast<int>(lim64);
        // the whole S row in registers: four loads in flight, one wait
        uint32_t s[kBN];
#pragma unroll
        for (int c4 = 0; c4 < kBN / 32; ++c4)
          tmem_ld32(tS + c4 * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c4 * 32]));
        tmem_wait_ld();
        if (!__all_sync(0xffffffffu, lim >= kBN - 1)) {
          // a key tile on the diagonal: keys past the row's position become -inf in
          // place, and the tile takes the same max and exponential code as a fully
          // visible one (the max ignores them; their P is 0 from ex2.approx, or
          // 2^-126 from the clamped polynomial: a weight of ~1e-38 against the row's
          // largest, 1).  A separate masked path, with its own max loop and selects
          // inside the exponentials, cost ~50 % more per step than a full tile.
#pragma unroll
          for (int c = 0; c < kBN; ++c) s[c] = c <= lim ? s[c] : 0xff800000u;
        }
        // four independent chains of three-input max: 43 instructions, short dependency chains
        float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
        for (int c = 0; c < kBN; c += 8) {
          m0 = max3f(m0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
          m1 = max3f(m1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
          m2 = max3f(m2, __uint_as_float(s[c + 4]), __uint_as_float(s[c + 5]));
          m3 = max3f(m3, __uint_as_float(s[c + 6]), __uint_as_float(s[c + 7]));
        }
        const float mx = max3f(m0, m1, fmaxf(m2, m3));
        const float m_tile = mx * sl2;
        float alpha = 1.f;
        bool rescale = false;
        if (j == 0) {
          m_used = m_tile;
        } else if (m_tile > m_used + 8.f) {
          alpha = ex2(m_used - m_tile);
          m_used = m_tile;
          rescale = true;
        }
        // O is rescaled before any P of this step is released, since PV(j) must see
        // it (O is stable: the commit behind this tile's S(j) covered PV(j-1))
        auto rescale_o = [&]() {
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(tO + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st32(tO + c * 32, o);
            }
          }
        };
        float ra0 = 0.f, ra1 = 0.f, rb0 = 0.f, rb1 = 0.f;   // packed partial row sums
        // a row with no visible key so far (m_used = -inf) has every key masked: a finite
        // offset keeps the masked arguments at -inf (ex2: 0) instead of NaN
        const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
#pragma unroll
        for (int c4 = 0; c4 < kBN / 32; ++c4) {
          uint32_t pk[16];
          exp_chunk<DT>(s, c4, sl2, neg_m, ra0, ra1, rb0, rb1, pk);
          // P chunk c4 -> columns [16 c4, 16 c4 + 16) (S was read completely above)
          tmem_st16(tS + c4 * 16, pk);
          if (kPvSplit && c4 == kBN / 64 - 1) {
            // keys 0-63 of P stored (their S registers are free for the rescale of O):
            // their PV may start
            rescale_o();
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_PHALF + t));
          }
        }
        const float rs = (ra0 + ra1) + (rb0 + rb1);
        l_sum = l_sum * alpha + rs;
        if (!kPvSplit) rescale_o();
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_PFULL + t));
      }
      if (failed) break;
      if (!__all_sync(0xffffffffu, wait_or_abort(bar(B_ODONE + t), oc & 1, abort_flag))) {
        failed = true;
        break;
      }
      ++oc;
      tc_fence_after();
      if (slot0 >= 0) {
        // split tile: this chunk's O / l (16-bit, the inputs' type), running max and row sum
        const int64_t slot = slot0 + ig.piece;
        uint16_t* po = prm.part_o + (slot * kBM + row) * HD;
        const float inv_l = l_sum > 0.f ? 1.f / l_sum : 0.f;   // no visible key: O = 0
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
          store_chunk<DT>(po + c * 32, o, inv_l, prm.store_v8);
        }
        prm.part_ml[slot * kBM + row] = make_float2(m_used, l_sum);
      } else {
        const float inv_l = 1.f / l_sum;
        const int hq = ig.kvh * prm.group + row % prm.group;
        uint16_t* orow = prm.out + (tok * prm.n_q_heads + hq) * static_cast<int64_t>(HD);
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
          if (row_valid) store_chunk<DT>(orow + c * 32, o, inv_l, prm.store_v8);
        }
      }
      // O has been read: the next item's first PV may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_OFREE + t));
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
// Work plan (one CTA).  A pair's steps are its later tile's 128-key tiles L_p
// (the earlier tile's La_p <= L_p are a prefix of them; L_p grows with p, the
// positions being ascending).  Every item also costs a fixed overhead of c0
// steps (Q load, pipeline refill, epilogue), so the plan balances
// steps + c0 * items over the SMs (B workers):
//   - small units (the longest, plus c0, at most half an SM's share): every
//     (KV head, pair) unit is one item, longest first, each item its own
//     worker: the dynamic queue then balances them like LPT scheduling, with
//     no split and nothing to merge;
//   - otherwise the units are laid end to end in cost space (c0, then the
//     unit's L_p steps) and cut into B equal ranges; a unit whose steps cross a
//     cut is split there into pieces (one item each), whose partial results
//     attn_combine_kernel merges.  A split unit's tiles get consecutive
//     partial slots: the earlier tile one per piece that holds some of its key
//     tiles (when more than one does), then the later tile one per piece.
// Items in unit order are grouped by worker; first_item[w] indexes them.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

// exclusive prefix sum over the block (1024 threads); *total receives the sum
__device__ int block_excl_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int w = s_warp[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    s_warp[lane] = wi - w;           // exclusive warp offsets
    if (lane == 31) s_warp[32] = wi;  // block total
  }
  __syncthreads();
  const int r = s_warp[warp] + x - v;
  *total = s_warp[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kPlanThreads, 1)
attn_plan_kernel(const int64_t* __restrict__ pos, int64_t n_sel, int tok_per_tile, int n_tiles,
                 int n_kv_heads, int target_workers, int item_cost, int max_items, int max_slots,
                 AttnPlanHeader* hdr, int4* items, int* first_item, int* pair_off, int* tile_base,
                 int4* split_desc, int32_t* status) {
  __shared__ int s_warp[33];
  __shared__ int s_error, s_lmax;
  const int tid = threadIdx.x;
  const int n_pairs = (n_tiles + 1) / 2;
  const int n_units = n_kv_heads * n_pairs;
  if (tid == 0) {
    s_error = 0;
    s_lmax = 0;
  }
  __syncthreads();
  auto tile_len = [&](int tile) {
    return tile >= 0 ? tile_key_tiles(pos, n_sel, n_tiles, tok_per_tile, tile) : 0;
  };
  // 1. pair step counts, their prefix (pair_off[p] = steps of pairs before p), the longest
  int carry = 0;
  for (int b0 = 0; b0 < n_pairs; b0 += kPlanThreads) {
    const int p = b0 + tid;
    int L = 0;
    if (p < n_pairs) {
      L = tile_len(pair_tile(n_tiles, p, 1));
      if (L > kMaxKvTiles) s_error = 1;
      atomicMax(&s_lmax, L);
    }
    int tot;
    const int off = block_excl_scan(L, s_warp, &tot);
    if (p < n_pairs) pair_off[p] = carry + off;
    carry += tot;
  }
  if (tid == 0) pair_off[n_pairs] = carry;
  __syncthreads();
  const int64_t Wh = carry;
  const int64_t W = Wh * n_kv_heads;                               // steps, >= 1
  const int64_t c0 = item_cost;
  const int64_t Wc = W + c0 * n_units;                             // cost
  const int64_t B = W < target_workers ? W : target_workers;

  if ((s_lmax + c0) * 2 * B <= Wc) {
    // ---- small units: one item each, longest first (pairs in descending order)
    if (n_units > max_items) s_error = 1;
    for (int i = tid; i < n_units && i < max_items; i += kPlanThreads) {
      const int p = n_pairs - 1 - i / n_kv_heads, h = i % n_kv_heads;
      items[i] = make_int4(h, p, 0, pair_off[p + 1] - pair_off[p]);
      first_item[i] = i;
    }
    for (int i = tid; i < n_kv_heads * n_tiles; i += kPlanThreads) tile_base[i] = -1;
    if (tid == 0) {
      const int n = n_units < max_items ? n_units : max_items;
      first_item[n] = n;
      hdr->n_items = n;
      hdr->n_workers = n;
      hdr->n_split = 0;
      hdr->n_slots = 0;
      hdr->error = s_error;
      hdr->next_item = 0;
      if (s_error) report(status, CBK_STATUS_COUNT);
    }
    return;
  }

  // ---- a dynamic tail: the shortest units (pairs p < p_cut, every head), about
  //      kAttnDynPct % of the cost, are whole items taken longest first by the CTAs
  //      that finish their static range early (each is a worker after the B static ones)
  if (tid == 0) s_lmax = 0;                                   // reused: p_cut
  __syncthreads();
  const int64_t dyn_budget = static_cast<int64_t>(kAttnDynPct) * Wc / 100;
  for (int p = 1 + tid; p < n_pairs; p += kPlanThreads)
    if (static_cast<int64_t>(n_kv_heads) * (pair_off[p] + c0 * p) <= dyn_budget) atomicMax(&s_lmax, p);
  __syncthreads();
  const int p_cut = s_lmax;
  const int n_ps = n_pairs - p_cut;                           // static pairs (>= 1)
  const int64_t Wh_s = Wh - pair_off[p_cut];
  const int64_t W_s = Wh_s * n_kv_heads;
  const int n_units_s = n_kv_heads * n_ps;
  const int64_t Wc_s = W_s + c0 * n_units_s;
  const int64_t Bs = W_s < target_workers ? W_s : target_workers;
  // ---- the static units as equal ranges of cost: unit u's steps are [Q_u, Q_u + L)
  //      in cost space, Q_u = (u + 1) c0 + P_u (P_u its first step in step space)
  auto worker_of = [&](int64_t x) { return ((x + 1) * Bs + Wc_s - 1) / Wc_s - 1; };
  auto worker_start = [&](int64_t w) { return w * Wc_s / Bs; };
  for (int64_t w = tid; w < Bs; w += kPlanThreads) first_item[w] = 0x7fffffff;
  __syncthreads();
  int item_carry = 0, slot_carry = 0, split_carry = 0;
  for (int b0 = 0; b0 < n_units_s; b0 += kPlanThreads) {
    const int u = b0 + tid;
    int n_pieces = 0, m_a = 0, ta = -1, tb = -1, L = 0, La = 0;
    int64_t Q = 0, wa = 0;
    if (u < n_units_s) {
      const int h = u / n_ps, p = p_cut + u % n_ps;
      ta = pair_tile(n_tiles, p, 0);
      tb = pair_tile(n_tiles, p, 1);
      L = pair_off[p + 1] - pair_off[p];
      La = tile_len(ta);
      Q = (u + 1) * c0 + h * Wh_s + (pair_off[p] - pair_off[p_cut]);
      wa = worker_of(Q);
      n_pieces = static_cast<int>(worker_of(Q + L - 1) - wa + 1);
      m_a = La > 0 ? static_cast<int>(worker_of(Q + La - 1) - wa + 1) : 0;
    }
    const int slots_a = m_a > 1 ? m_a : 0, slots_b = n_pieces > 1 ? n_pieces : 0;
    int tot_items, tot_slots, tot_split;
    const int item0 = item_carry + block_excl_scan(n_pieces, s_warp, &tot_items);
    const int slot0 = slot_carry + block_excl_scan(slots_a + slots_b, s_warp, &tot_slots);
    const int split0 = split_carry + block_excl_scan((slots_a > 0) + (slots_b > 0), s_warp, &tot_split);
    if (u < n_units_s) {
      const int h = u / n_ps, p = p_cut + u % n_ps;
      for (int i = 0; i < n_pieces; ++i) {
        const int64_t w = wa + i;
        const int64_t sw = worker_start(w), sw1 = worker_start(w + 1);
        const int j0 = static_cast<int>((sw > Q ? sw : Q) - Q);
        const int j1 = static_cast<int>((sw1 < Q + L ? sw1 : Q + L) - Q);
        const int at = item0 + i;
        if (at < max_items) items[at] = make_int4(h, p, j0, j1 | (i << 16));
        atomicMin(&first_item[w], at);
      }
      if (ta >= 0) tile_base[h * n_tiles + ta] = slots_a ? slot0 : -1;
      tile_base[h * n_tiles + tb] = slots_b ? slot0 + slots_a : -1;
      int sp = split0;
      if (slots_a) split_desc[sp++] = make_int4(h * n_tiles + ta, slot0, slots_a, 0);
      if (slots_b) split_desc[sp] = make_int4(h * n_tiles + tb, slot0 + slots_a, slots_b, 0);
    }
    item_carry += tot_items;
    slot_carry += tot_slots;
    split_carry += tot_split;
  }
  // the dynamic units: whole, pairs p_cut - 1 down to 0, each its own worker
  const int n_dyn = n_kv_heads * p_cut;
  for (int i = tid; i < n_dyn; i += kPlanThreads) {
    const int p = p_cut - 1 - i / n_kv_heads, h = i % n_kv_heads;
    const int at = item_carry + i;
    if (at < max_items) items[at] = make_int4(h, p, 0, pair_off[p + 1] - pair_off[p]);
    first_item[Bs + i] = at;
    const int ta = pair_tile(n_tiles, p, 0), tb = pair_tile(n_tiles, p, 1);
    if (ta >= 0) tile_base[h * n_tiles + ta] = -1;
    tile_base[h * n_tiles + tb] = -1;
  }
  __syncthreads();
  if (tid == 0) {
    const int n_items = item_carry + n_dyn;
    if (n_items > max_items || slot_carry > max_slots) s_error = 1;
    // a static worker whose range holds no step (it fell inside items' overheads) has no items
    first_item[Bs + n_dyn] = n_items;
    if (n_dyn == 0) first_item[Bs] = item_carry;
    for (int64_t w = Bs - 1; w >= 0; --w)
      if (first_item[w] == 0x7fffffff) first_item[w] = first_item[w + 1];
    hdr->n_items = n_items;
    hdr->n_workers = static_cast<int>(Bs) + n_dyn;
    hdr->n_split = split_carry;
    hdr->n_slots = slot_carry;
    hdr->error = s_error;
    hdr->next_item = 0;
    if (s_error) report(status, CBK_STATUS_COUNT);
  }
}

// ---------------------------------------------------------------------------
// Merge the partial results of split tiles:
//   O = sum_c w_c Ohat_c / sum_c w_c,  w_c = l_c 2^(m_c - M),  Ohat_c = O_c / l_c
// (a chunk without visible keys has l = 0 and weight 0).  Work unit = a quarter
// of a split tile (32 rows), one CTA of 128 threads; a thread owns kVecThr
// 8-element vectors of different rows and computes those rows' maxima and
// weights itself from the (m, l) pairs (no shared memory, no block barriers).
// The first kCombinePre chunks' O vectors and (m, l) pairs are loaded together,
// so a unit of up to kCombinePre chunks costs one round trip to L2; small units
// and few registers let every unit of a call have its own resident CTA.  Sums run
// over the chunks in increasing order, so results are deterministic.
// ---------------------------------------------------------------------------
constexpr int kCombineThreads = 128;
constexpr int kCombineRows = 32;        // rows per work unit
constexpr int kCombinePre = 2;          // chunk rows loaded together (most split tiles have two)

template <int DT, int HD>
__global__ void __launch_bounds__(kCombineThreads, 5)
attn_combine_kernel(const AttnParams prm) {
  constexpr int kVecRow = HD / 8;                                     // 8-element vectors per row
  constexpr int kVecThr = kCombineRows * kVecRow / kCombineThreads;  // 4 (HD 128) or 2 (HD 64)
  constexpr int kRowStep = kCombineThreads / kVecRow;                 // rows between a thread's vectors
  const int tid = threadIdx.x;
  // launched as a programmatic dependent of the attention kernel: wait until that
  // grid has finished and its partial results are visible (a no-op otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every attention CTA has finished: rewind the item queue for the next call
  if (blockIdx.x == 0 && tid == 0) *prm.queue = 0;
  if (prm.plan->error) return;
  const int n_units = prm.plan->n_split * (kBM / kCombineRows);
  const int v = tid % kVecRow;                   // the thread's vector within each of its rows
  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int4 d = prm.split_desc[u / (kBM / kCombineRows)];
    const int row0 = (u % (kBM / kCombineRows)) * kCombineRows + tid / kVecRow;   // row of vector 0
    const int kvh = d.x / prm.n_tiles, tile = d.x % prm.n_tiles;
    const int64_t slot0 = d.y;
    const int nc = d.z;
    auto o_ptr = [&](int c, int i) {
      return prm.part_o + ((slot0 + c) * kBM + row0 + i * kRowStep) * HD + v * 8;
    };
    auto ml_ptr = [&](int c, int i) { return prm.part_ml + (slot0 + c) * kBM + row0 + i * kRowStep; };
    uint4 raw[kCombinePre][kVecThr];
    float2 mlp[kCombinePre][kVecThr];
#pragma unroll
    for (int q = 0; q < kCombinePre; ++q)
      if (q < nc) {
#pragma unroll
        for (int i = 0; i < kVecThr; ++i) {
          raw[q][i] = ld_vec(o_ptr(q, i));
          mlp[q][i] = *ml_ptr(q, i);
        }
      }
    float M[kVecThr];
#pragma unroll
    for (int i = 0; i < kVecThr; ++i) M[i] = -INFINITY;
#pragma unroll
    for (int q = 0; q < kCombinePre; ++q)
      if (q < nc) {
#pragma unroll
        for (int i = 0; i < kVecThr; ++i)
          if (mlp[q][i].y > 0.f) M[i] = fmaxf(M[i], mlp[q][i].x);
      }
    for (int c = kCombinePre; c < nc; ++c)
#pragma unroll
      for (int i = 0; i < kVecThr; ++i) {
        const float2 ml = *ml_ptr(c, i);
        if (ml.y > 0.f) M[i] = fmaxf(M[i], ml.x);
      }
    float acc[kVecThr][8], sum[kVecThr];
#pragma unroll
    for (int i = 0; i < kVecThr; ++i) {
      sum[i] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
    }
    for (int c0 = 0; c0 < nc; c0 += kCombinePre) {
      if (c0 > 0) {
#pragma unroll
        for (int q = 0; q < kCombinePre; ++q)
          if (c0 + q < nc) {
#pragma unroll
            for (int i = 0; i < kVecThr; ++i) raw[q][i] = ld_vec(o_ptr(c0 + q, i));
          }
      }
#pragma unroll
      for (int q = 0; q < kCombinePre; ++q)
        if (c0 + q < nc) {
#pragma unroll
          for (int i = 0; i < kVecThr; ++i) {
            const float2 ml = c0 == 0 ? mlp[q][i] : *ml_ptr(c0 + q, i);
            const float w = ml.y > 0.f ? ml.y * ex2(ml.x - M[i]) : 0.f;
            sum[i] += w;
            const uint16_t* h = reinterpret_cast<const uint16_t*>(&raw[q][i]);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[i][e] = fmaf(w, Elem<DT>::to_f(h[e]), acc[i][e]);
          }
        }
    }
#pragma unroll
    for (int i = 0; i < kVecThr; ++i) {
      const int row = row0 + i * kRowStep;
      const int64_t tok = tile_tok0(prm.n_sel, prm.n_tiles, prm.tok_per_tile, tile) + row / prm.group;
      if (tok < 0) continue;             // padding row of the first tile
      const float inv = 1.f / sum[i];
      const int hq = kvh * prm.group + row % prm.group;
      uint4 o;
      uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = pack2<DT>(acc[i][2 * e] * inv, acc[i][2 * e + 1] * inv);
      st_vec(prm.out + (tok * prm.n_q_heads + hq) * static_cast<int64_t>(HD) + v * 8, o);
    }
  }
}

// ---------------------------------------------------------------------------
// host side: tensor maps, workspace layout, launch
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

static int sm_count() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Workspace layout of one partial-attention call (all offsets 256-byte aligned).
struct AttnLayout {
  int tok_per_tile, n_tiles, n_pairs, target, max_items, max_slots;
  size_t off_items, off_first, off_pair, off_tile_base, off_split, off_ml, off_o, bytes;
};

static size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }


static AttnLayout attn_layout(int64_t n_sel, int n_q_heads, int n_kv_heads, int head_dim) {
  AttnLayout a;
  const int G = n_q_heads / n_kv_heads;
  a.tok_per_tile = kBM / G;
  a.n_tiles = static_cast<int>((n_sel + a.tok_per_tile - 1) / a.tok_per_tile);
  a.n_pairs = (a.n_tiles + 1) / 2;
  a.target = kAttnWorkersPerSm * sm_count();   // workers: equal ranges of cost, per SM
  // items: one per unit plus one per worker boundary inside a unit
  a.max_items = a.target + n_kv_heads * a.n_pairs;
  // a split unit holds a worker boundary, so split units' pieces number <= 2 (workers - 1),
  // and each piece gives at most two slots (earlier and later tile)
  a.max_slots = 4 * a.target + 2;
  a.off_items = align256(sizeof(AttnPlanHeader));
  a.off_first = a.off_items + align256(static_cast<size_t>(a.max_items) * sizeof(int4));
  a.off_pair = a.off_first + align256(static_cast<size_t>(a.max_items + 1) * sizeof(int));
  a.off_tile_base = a.off_pair + align256(static_cast<size_t>(a.n_pairs + 1) * sizeof(int));
  a.off_split = a.off_tile_base + align256(static_cast<size_t>(n_kv_heads) * a.n_tiles * sizeof(int));
  a.off_ml = a.off_split + align256(static_cast<size_t>(n_kv_heads) * a.n_tiles * sizeof(int4));
  a.off_o = a.off_ml + align256(static_cast<size_t>(a.max_slots) * kBM * sizeof(float2));
  a.bytes = a.off_o + static_cast<size_t>(a.max_slots) * kBM * head_dim * sizeof(uint16_t);
  return a;
}

// resident CTAs of attn_combine_kernel per SM (occupancy of its registers), cached
template <int DT, int HD>
static int combine_ctas_per_sm() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  if (!cache[dev]) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_combine_kernel<DT, HD>, kCombineThreads, 0) !=
            cudaSuccess ||
        n <= 0)
      n = 1;
    cache[dev] = n;
  }
  return cache[dev];
}

template <int DT, int HD>
static int launch_attn(const void* q, const void* k, const void* v, const int64_t* pos,
                       int64_t n_sel, int64_t S, int n_q_heads, int n_kv_heads, float scale,
                       void* out, void* workspace, int reuse_plan, int32_t* status, cudaStream_t st) {
  const int G = n_q_heads / n_kv_heads;
  const AttnLayout lay = attn_layout(n_sel, n_q_heads, n_kv_heads, HD);
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, q, DT, HD, n_q_heads, n_sel, G, kBM / G)) return rc;
  if (int rc = make_map(&mk, k, DT, HD, n_kv_heads, S, 1, kBN)) return rc;
  if (int rc = make_map(&mv, v, DT, HD, n_kv_heads, S, 1, kBN)) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  AttnParams prm;
  prm.pos = pos;
  prm.out = static_cast<uint16_t*>(out);
  prm.status = status;
  prm.plan = reinterpret_cast<const AttnPlanHeader*>(ws);
  prm.queue = &reinterpret_cast<AttnPlanHeader*>(ws)->next_item;
  prm.items = reinterpret_cast<const int4*>(ws + lay.off_items);
  prm.first_item = reinterpret_cast<const int*>(ws + lay.off_first);
  prm.tile_base = reinterpret_cast<const int*>(ws + lay.off_tile_base);
  prm.split_desc = reinterpret_cast<const int4*>(ws + lay.off_split);
  prm.part_ml = reinterpret_cast<float2*>(ws + lay.off_ml);
  prm.part_o = reinterpret_cast<uint16_t*>(ws + lay.off_o);
  prm.n_sel = n_sel;
  prm.n_q_heads = n_q_heads;
  prm.group = G;
  prm.tok_per_tile = lay.tok_per_tile;
  prm.n_tiles = lay.n_tiles;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.store_v8 = ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(workspace)) & 31u) == 0;
  if (!reuse_plan) {
    attn_plan_kernel<<<1, kPlanThreads, 0, st>>>(
        pos, n_sel, lay.tok_per_tile, lay.n_tiles, n_kv_heads, lay.target, kAttnItemCost, lay.max_items,
        lay.max_slots,
        reinterpret_cast<AttnPlanHeader*>(ws), reinterpret_cast<int4*>(ws + lay.off_items),
        reinterpret_cast<int*>(ws + lay.off_first), reinterpret_cast<int*>(ws + lay.off_pair),
        reinterpret_cast<int*>(ws + lay.off_tile_base), reinterpret_cast<int4*>(ws + lay.off_split), status);
    if (int rc = check_launch("attn_plan_kernel")) return rc;
  }
  auto kern = partial_attn_kernel<DT, HD>;
  const int smem = AttnSmem<HD>::kAlloc;
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem)) return rc;
  const int grid = sm_count();             // persistent: one CTA per SM, taking workers from the queue
  kern<<<static_cast<unsigned>(grid), kThreads, smem, st>>>(mq, mk, mv, prm);
  if (int rc = check_launch("partial_attn_kernel")) return rc;
  // one CTA per half split tile; at most every tile is split.  One wave: no more
  // CTAs than fit on the GPU at once (the plan's split tiles are not known on the
  // host; CTAs past the plan's units exit at once, the others loop over units)
  const int64_t max_units = static_cast<int64_t>(n_kv_heads) * lay.n_tiles * (kBM / kCombineRows);
  const int comb_grid = static_cast<int>(std::min<int64_t>(max_units, combine_ctas_per_sm<DT, HD>() * sm_count()));
  // programmatic dependent launch: the merge kernel's CTAs can be placed on SMs the
  // attention kernel has left (each attention CTA signals when the queue is empty)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(comb_grid));
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_combine_kernel<DT, HD>, prm);
  if (e != cudaSuccess) return set_error(CBK_ERR_CUDA, "attn_combine_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("attn_combine_kernel");
}

}  // namespace cbk

using namespace cbk;

static int check_attn_geometry(int n_q_heads, int n_kv_heads, int head_dim, int64_t n_sel, int64_t S) {
  if (head_dim != 64 && head_dim != 128)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_partial_attn: head_dim %d (64 or 128 only)", head_dim);
  if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads != 0)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: n_q_heads must be a multiple of n_kv_heads");
  const int G = n_q_heads / n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_partial_attn: GQA group %d not in {1,2,4,8,16}", G);
  if (S <= 0 || n_sel < 0 || S > static_cast<int64_t>(kMaxKvTiles - 1) * kBN || n_sel > S)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: need 0 <= n_sel <= S <= %d (n_sel %lld, S %lld)",
                     (kMaxKvTiles - 1) * kBN, (long long)n_sel, (long long)S);
  return CBK_OK;
}

extern "C" size_t cbk_partial_attn_workspace_bytes(int64_t n_sel, int64_t S, int n_q_heads,
                                                   int n_kv_heads, int head_dim) {
  if (check_attn_geometry(n_q_heads, n_kv_heads, head_dim, n_sel, S) != CBK_OK) return 0;
  return attn_layout(n_sel < 1 ? 1 : n_sel, n_q_heads, n_kv_heads, head_dim).bytes;
}

extern "C" int cbk_partial_attn(const void* q, const void* k, const void* v, const int64_t* pos,
                                int64_t n_sel, int64_t S, int n_q_heads, int n_kv_heads,
                                int head_dim, float scale, int dtype, void* out, void* workspace,
                                size_t workspace_bytes, int reuse_plan, int32_t* status,
                                void* stream) {
  if (dtype != CBK_BF16 && dtype != CBK_F16)
    return set_error(CBK_ERR_UNSUPPORTED, "cbk_partial_attn: dtype %d not supported", dtype);
  if (int rc = check_attn_geometry(n_q_heads, n_kv_heads, head_dim, n_sel, S)) return rc;
  if (!q || !k || !v || !pos || !out || !workspace)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(workspace)) & 15u)
    return set_error(CBK_ERR_INVALID, "cbk_partial_attn: q/k/v/out/workspace must be 16-byte aligned");
  if (n_sel == 0) return CBK_OK;
  const size_t need = attn_layout(n_sel, n_q_heads, n_kv_heads, head_dim).bytes;
  if (workspace_bytes < need)
    return set_error(CBK_ERR_WORKSPACE, "cbk_partial_attn: workspace %zu < %zu bytes", workspace_bytes, need);
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == CBK_BF16)
    return head_dim == 128
               ? launch_attn<CBK_BF16, 128>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, workspace, reuse_plan, status, st)
               : launch_attn<CBK_BF16, 64>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, workspace, reuse_plan, status, st);
  return head_dim == 128
             ? launch_attn<CBK_F16, 128>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, workspace, reuse_plan, status, st)
             : launch_attn<CBK_F16, 64>(q, k, v, pos, n_sel, S, n_q_heads, n_kv_heads, scale, out, workspace, reuse_plan, status, st);
}

