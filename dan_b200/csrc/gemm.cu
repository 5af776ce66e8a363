// Dense projections on the 5th-generation tensor cores: C = A * W^T.
//
// A [M, K] (activations, K-major) and W [N, K] (nn.Linear weight, K-major) are
// staged by TMA into a 4-deep ring of 128-byte-swizzled shared-memory tiles;
// one elected thread issues tcgen05.mma (128 x 256 x 16 bf16, or 128 x 256 x 32
// e4m3) accumulating in TMEM; four epilogue warps read the fp32 accumulator
// back with tcgen05.ld and apply the fused epilogue. The kernel is persistent
// (one CTA per SM, tiles strided by the grid) and double-buffers the TMEM
// accumulator (2 x 256 columns) so the epilogue of tile i overlaps the main
// loop of tile i+1. For M >= 256 a CTA-pair variant computes 256 x 256 tiles
// in a grouped order that keeps the smaller operand's slice resident in L2,
// and splits the last ragged wave of deep (>= 128 K iterations) tiles by K
// across all pairs (stream-K, partial sums reduced in a fixed order); a ragged
// last wave of shallower tiles runs as narrow column slices on the idle pairs.
// Each epilogue warp stages 32 x 32 output chunks in shared memory and sends
// them with TMA stores (the residual arrives by TMA load the same way).
//
// Epilogues (replacing separate passes of the reference):
//   store     C = bf16(acc [+ bias])                          (nn.Linear, llama.py:78,102)
//   residual  C = bf16(R + bf16(acc [+ bias]))                (x + o_proj(...), llama.py:116-117)
//   swiglu    W rows interleaved in 128-row blocks [gate | up]; C[:, j] = bf16(silu(g) * u)
//             with g, u the bf16-rounded projections          (fused.py:59-61, llama.py:100-103)
// The e4m3 variant multiplies acc by a_scale[row] * w_scale[col] first
// (torch._scaled_mm with row-wise scales, quant.py:37-42).
#include "common.cuh"

#include <map>
#include <mutex>

namespace dan {
namespace gemm {

constexpr int BM = 128, BN = 256;
constexpr int KBYTES = 128;  // bytes of K per stage (one 128 B swizzle row)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * KBYTES;
constexpr int B_BYTES = BN * KBYTES;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int SMEM_BYTES_BASE = STAGES * STAGE_BYTES + 1024 + 512;  // + the epilogue sink

enum Epilogue { kStore = 0, kResidual = 1, kSwiglu = 2, kRope = 3 };

struct Params {
  __nv_bfloat16* c;
  int64_t ldc;
  const __nv_bfloat16* resid;
  int64_t ldr;
  const __nv_bfloat16* bias;
  const float* a_scale;  // e4m3 only: per row of A
  const float* w_scale;  // e4m3 only: per row of W (output channel)
  int m, n, k;
  int tiles_m, tiles_n;
  int epilogue;
  int rope_cols;        // kRope: leading output columns holding rotary heads
  int rope_hd;          // kRope: head size (64, 128 or 256); pairs (i, i + hd/2) rotate
  const float* cos_t;   // kRope: [m, hd/2] bf16-rounded cos of each row's angles
  const float* sin_t;
  int32_t* status;
  int order;    // pair kernel tile order: 0 = m fastest (A stays in L2), 1 = n fastest (W stays)
  int group;    // pair kernel: tile rows (order 0) or columns (order 1) per raster group
  // Stream-K (pair kernel): tiles [sk_first, tiles) are split by K iteration across the pairs,
  // sk_iters iterations in all; 0 = every tile whole.
  int sk_first, sk_iters;
  // Narrow tail (pair kernel, no stream-K): tiles [nt_first, sk_first) each run as nt_split
  // items of BN / nt_split columns, so a ragged last wave spreads over more pairs; 1 = none.
  int nt_first, nt_split;
  float* sk_part;                 // [pairs][2 ranks][2 segments][BN][128] fp32 partials, column-major
  unsigned long long* sk_cnt;     // [2 pairs][2 ranks][4 warps] arrivals per split tile: epoch << 32 | n
  uint32_t* sk_ctrl;              // [0] epoch, [1] CTAs finished in this launch
  int tma_out;        // epilogue writes through the shared-memory sink and TMA stores
};

constexpr int64_t kGroupBytes = 32LL << 20;

// Tile t of the pair kernel's sequence. Tiles run in groups of ``group`` rows (order 0) or
// columns (order 1) of the tile grid; inside a group the grouped dimension varies fastest, so
// each wave re-touches the group's stationary operand slice and streams the other operand.
__device__ __forceinline__ void pair_tile(int t, int tiles_m, int tiles_n, int order, int group, int& tm,
                                          int& tn) {
  const int gdim = order == 0 ? tiles_m : tiles_n, odim = order == 0 ? tiles_n : tiles_m;
  const int per = group * odim;
  const int g = t / per, r = t - g * per;
  const int first = g * group;
  const int span = gdim - first < group ? gdim - first : group;
  const int a = first + r % span, b = r / span;
  tm = order == 0 ? a : b;
  tn = order == 0 ? b : a;
}

// One unit of a pair's work: K iterations [kb, ke) of tile t, restricted to column slice ``sub``
// of ``width`` columns (width BN: the whole tile).
struct PairItem {
  int t, kb, ke, sub, width;
};

// The pair kernel's work list: items pair, pair + P, ... of the data-parallel list (whole tiles
// below nt_first, then nt_split narrow items per tile up to sk_first), then this pair's
// contiguous share [g, g1) of the stream-K iterations, cut at tile boundaries into segments.
// A pair's share is contiguous, so only its first segment can start inside a tile and only
// its last can stop inside one.
struct PairWork {
  int next_dp, dp_items, dp_end, nt_first, ns, n_pairs, k_iters, g, g1;
  __device__ __forceinline__ PairWork(int pair, int P, const Params& p, int ki)
      : next_dp(pair),
        dp_items(p.nt_first + (p.sk_first - p.nt_first) * p.nt_split),
        dp_end(p.sk_first),
        nt_first(p.nt_first),
        ns(p.nt_split),
        n_pairs(P),
        k_iters(ki) {
    g = static_cast<int>(static_cast<long long>(pair) * p.sk_iters / P);
    g1 = static_cast<int>(static_cast<long long>(pair + 1) * p.sk_iters / P);
  }
  __device__ __forceinline__ bool next(PairItem& w) {
    w.sub = 0;
    w.width = BN;
    if (next_dp < dp_items) {
      const int it = next_dp;
      next_dp += n_pairs;
      if (it < nt_first) {
        w.t = it;
      } else {
        const int j = it - nt_first, q = j / ns;
        w.t = nt_first + q;
        w.sub = j - q * ns;
        w.width = BN / ns;
      }
      w.kb = 0;
      w.ke = k_iters;
      return true;
    }
    if (g >= g1) return false;
    const int tr = g / k_iters;
    w.t = dp_end + tr;
    w.kb = g - tr * k_iters;
    w.ke = w.kb + (g1 - g) < k_iters ? w.kb + (g1 - g) : k_iters;
    g += w.ke - w.kb;
    return true;
  }
};

// e4m3 epilogues: scale the 32 accumulators of one chunk in place by a_scale[row] *
// w_scale[col + i] (0 past n) before the element loop: eight 16-byte loads of the scales when
// the chunk is whole and aligned (one uniform branch per chunk, none per element).
__device__ __forceinline__ void scale_chunk(const Params& p, int col, float as, uint32_t (&r)[32]) {
  if (col + 32 <= p.n && (reinterpret_cast<uintptr_t>(p.w_scale + col) & 15) == 0) {
    const float4* w4 = reinterpret_cast<const float4*>(p.w_scale + col);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = __ldg(w4 + j);
      r[4 * j] = __float_as_uint(__uint_as_float(r[4 * j]) * (as * w.x));
      r[4 * j + 1] = __float_as_uint(__uint_as_float(r[4 * j + 1]) * (as * w.y));
      r[4 * j + 2] = __float_as_uint(__uint_as_float(r[4 * j + 2]) * (as * w.z));
      r[4 * j + 3] = __float_as_uint(__uint_as_float(r[4 * j + 3]) * (as * w.w));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      r[i] = __float_as_uint(__uint_as_float(r[i]) * (as * (col + i < p.n ? p.w_scale[col + i] : 0.f)));
  }
}

// e4m3: the tile's 256 weight scales, lane l holding columns l, l + 32, ... (loaded before the
// epilogue waits for the accumulator, so their latency hides behind the main loop), and the
// register of 32-column group k (uniform) for a broadcast by shuffle.
__device__ __forceinline__ void load_tile_scales(const Params& p, int tn, int lane, float (&ws)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = tn * BN + 32 * j + lane;
    ws[j] = col < p.n ? p.w_scale[col] : 0.f;
  }
}
__device__ __forceinline__ float pick8(const float (&w)[8], int k) {
  float r = w[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) r = k == j ? w[j] : r;
  return r;
}

__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t x) { return *reinterpret_cast<__nv_bfloat162*>(&x); }
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 x) { return *reinterpret_cast<uint32_t*>(&x); }

template <bool FP8>
__device__ __forceinline__ void store_chunk(const Params& p, int row, int col, int cols_out, const float* v) {
  // v: 32 consecutive output values of ``row`` starting at ``col``.
  if (row >= p.m) return;
  __nv_bfloat16* dst = p.c + static_cast<int64_t>(row) * p.ldc + col;
  uint32_t packed[16];
  const bool full = col + 32 <= cols_out && (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
  if (p.epilogue == kResidual) {
    const __nv_bfloat16* r = p.resid + static_cast<int64_t>(row) * p.ldr + col;
    if (full && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
      uint4 rv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rv[i] = reinterpret_cast<const uint4*>(r)[i];
      const uint32_t* r2 = reinterpret_cast<const uint32_t*>(rv);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        packed[i] = as_u32(__hadd2_rn(as_bf2(r2[i]), as_bf2(pack_bf16(v[2 * i], v[2 * i + 1]))));
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float a = 0.f, b = 0.f;
        if (col + 2 * i < cols_out) a = __bfloat162float(r[2 * i]);
        if (col + 2 * i + 1 < cols_out) b = __bfloat162float(r[2 * i + 1]);
        packed[i] = pack_bf16(a + bf16_round(v[2 * i]), b + bf16_round(v[2 * i + 1]));
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) packed[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
  }
  if (full) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
  } else {  // ragged edge or unaligned row: element stores (constant indices keep packed[] in registers)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (col + 2 * i < cols_out) dst[2 * i] = __ushort_as_bfloat16(static_cast<unsigned short>(packed[i] & 0xffffu));
      if (col + 2 * i + 1 < cols_out) dst[2 * i + 1] = __ushort_as_bfloat16(static_cast<unsigned short>(packed[i] >> 16));
    }
  }
}

// Output path of one epilogue warp. With ``tma`` set (C, and R for the residual epilogue, are
// 16-byte aligned with 16-byte row pitch) each 32-row x 32-column bf16 chunk is written to one
// of the warp's four 2 KB shared-memory slots and leaves by a TMA store, which writes whole
// lines and clips rows >= m and columns >= the output width; the residual of a chunk arrives
// in its slot by TMA load one chunk ahead. Otherwise every thread stores its own row.
struct Sink {
  bool tma;
  uint8_t* stage;  // this warp's 4 slots of 32 rows x 64 bytes
  uint64_t* bar;   // this warp's 4 residual-load barriers
  const CUtensorMap* tc;
  const CUtensorMap* tr;
  uint32_t seq;    // chunks this warp has sent so far (slot = seq % 4)
  uint32_t phase;  // bit s: parity of slot s's next residual-load completion
  int row0;        // first output row of this warp's 32 rows in the current tile
  int lane;
  int m;           // rows of C: a warp whose rows all lie at or past m sends nothing
};

constexpr int SLOT_BYTES = 32 * 64;
constexpr int SINK_BYTES = 4 * 4 * SLOT_BYTES;  // 4 epilogue warps x 4 slots

__device__ __forceinline__ void pack32(const float* v, uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
}

// Send one packed chunk (this lane's 32 values of row row0 + lane, columns [col, col + 32)).
__device__ __forceinline__ void sink_put(Sink& o, int col, const uint32_t (&pk)[16]) {
  if (o.row0 >= o.m) return;
  uint8_t* slot = o.stage + (o.seq & 3) * SLOT_BYTES;
  if (o.lane == 0) bulk_wait_read<3>();  // the store sent from this slot four chunks ago has read it
  __syncwarp();
  uint4* d = reinterpret_cast<uint4*>(slot + o.lane * 64);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
  fence_proxy_async();
  __syncwarp();
  if (o.lane == 0) {
    tma_store_2d(o.tc, slot, col, o.row0);
    bulk_commit();
  }
  __syncwarp();  // reconverge before the next warp-collective tcgen05.ld
  ++o.seq;
}

// Write 32 epilogue values of one row: through the sink, or directly (store_chunk).
template <bool FP8>
__device__ __forceinline__ void emit(Sink& o, const Params& p, int row, int col, int cols_out, const float* v) {
  if (o.tma) {
    uint32_t pk[16];
    pack32(v, pk);
    sink_put(o, col, pk);
  } else {
    store_chunk<FP8>(p, row, col, cols_out, v);
  }
}

// Write 32 packed bf16 values (16 pairs) of one row: through the sink, or direct stores.
__device__ __forceinline__ void emit_packed(Sink& o, const Params& p, int row, int col, int cols_out,
                                            const uint32_t (&pk)[16]) {
  if (o.tma) {
    sink_put(o, col, pk);
    return;
  }
  if (row >= p.m) return;
  __nv_bfloat16* dst = p.c + static_cast<int64_t>(row) * p.ldc + col;
  if (col + 32 <= cols_out && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (col + 2 * i < cols_out) dst[2 * i] = __ushort_as_bfloat16(static_cast<unsigned short>(pk[i] & 0xffffu));
      if (col + 2 * i + 1 < cols_out) dst[2 * i + 1] = __ushort_as_bfloat16(static_cast<unsigned short>(pk[i] >> 16));
    }
  }
}

__device__ __forceinline__ void sink_load_resid(Sink& o, uint32_t seq, int col) {
  const uint32_t s = seq & 3;
  mbar_expect_tx(&o.bar[s], SLOT_BYTES);
  tma_load_2d(o.stage + s * SLOT_BYTES, o.tr, &o.bar[s], col, o.row0);
}

// Residual epilogue through the sink: C = bf16(R + bf16(acc [+ bias])) chunk by chunk, the
// next chunk's residual loading while this one is computed.
template <bool FP8>
__device__ __forceinline__ void residual_tma(Sink& o, const Params& p, uint32_t taddr, int col0, int cols,
                                             float as) {
  if (o.row0 >= p.m) return;
  const int width = p.n - col0 < cols ? p.n - col0 : cols;
  const int nch = (width + 31) / 32;
  if (o.lane == 0) {
    bulk_wait_read<3>();
    sink_load_resid(o, o.seq, col0);
  }
  __syncwarp();
#pragma unroll 1
  for (int i = 0; i < nch; ++i) {
    const int col = col0 + 32 * i;
    const uint32_t s = o.seq & 3;
    uint32_t r[32];
    tmem_ld32(taddr + 32 * i, r);
    if (o.lane == 0 && i + 1 < nch) {
      bulk_wait_read<2>();  // the slot the next residual lands in has been read by its last store
      sink_load_resid(o, o.seq + 1, col + 32);
    }
    __syncwarp();
    tmem_wait_ld_regs(r);
    if (FP8) scale_chunk(p, col, as, r);
    if (!mbar_wait(&o.bar[s], (o.phase >> s) & 1u)) report(p.status, kTimeoutFull);
    o.phase ^= 1u << s;
    uint4* slot = reinterpret_cast<uint4*>(o.stage + s * SLOT_BYTES + o.lane * 64);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 q = slot[g];
      uint32_t pk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = 8 * g + 2 * j;
        float x0 = __uint_as_float(r[c]), x1 = __uint_as_float(r[c + 1]);
        if (p.bias) {
          x0 += col + c < p.n ? __bfloat162float(p.bias[col + c]) : 0.f;
          x1 += col + c + 1 < p.n ? __bfloat162float(p.bias[col + c + 1]) : 0.f;
        }
        // bf16(R + bf16(acc)) as one rounded bf16 add (the sum of two bf16 values rounds the
        // same whether or not it passes through fp32 first)
        pk[j] = as_u32(__hadd2_rn(as_bf2((&q.x)[j]), as_bf2(pack_bf16(x0, x1))));
      }
      slot[g] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    fence_proxy_async();
    __syncwarp();
    if (o.lane == 0) {
      tma_store_2d(o.tc, o.stage + s * SLOT_BYTES, col, o.row0);
      bulk_commit();
    }
    __syncwarp();
    ++o.seq;
  }
}

// Pull the row's RoPE cos / sin into L2 while the tile's main loop still runs.
__device__ __forceinline__ void epilogue_prefetch(const Params& p, int row, int tn) {
  if (row >= p.m || p.epilogue != kRope || tn * BN >= p.rope_cols) return;
  const int half = p.rope_hd / 2;
  const char* c = reinterpret_cast<const char*>(p.cos_t + static_cast<int64_t>(row) * half);
  const char* s = reinterpret_cast<const char*>(p.sin_t + static_cast<int64_t>(row) * half);
  for (int b = 0; b < half * 4; b += 128) {
    prefetch_l2(c + b);
    prefetch_l2(s + b);
  }
}

// The fused epilogue of one 128-row accumulator held in TMEM at ``taddr`` (this warp's lanes):
// ``row`` is this thread's output row, ``tn`` the tile's column block, and the accumulator
// holds column slice ``sub`` of ``width`` columns of that block (width BN: the whole block).
// A slice is contiguous, except for SwiGLU, where it is width / 2 gate columns followed by
// the same width / 2 up columns (each CTA of the pair stages one half of W's rows).
template <bool FP8>
__device__ __forceinline__ void epilogue_tile(const Params& p, Sink& o, uint32_t taddr, int row, int tn, int sub,
                                              int width, const float (&ws)[8]) {
  const int cols_out = p.epilogue == kSwiglu ? p.n / 2 : p.n;
  const float as = (FP8 && row < p.m) ? p.a_scale[row] : 1.f;
  if (p.epilogue == kSwiglu) {
    const int half = width / 2, off = sub * half;
#pragma unroll 1
    for (int c = 0; c < half; c += 32) {
      uint32_t g[32], u[32];
      tmem_ld32(taddr + c, g);
      tmem_ld32(taddr + half + c, u);
      tmem_wait_ld();
      const int gcol = tn * BN + off + c, ucol = tn * BN + BN / 2 + off + c;
      if (FP8) {
        scale_chunk(p, gcol, as, g);
        scale_chunk(p, ucol, as, u);
      }
      // The reference's rounding points (fused.py:59-61 on bf16 projections): gate and up
      // rounded to bf16, silu(gate) rounded to bf16, then one rounded bf16 product.
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float g0 = __uint_as_float(g[2 * i]), g1 = __uint_as_float(g[2 * i + 1]);
        float u0 = __uint_as_float(u[2 * i]), u1 = __uint_as_float(u[2 * i + 1]);
        if (p.bias) {
          g0 += gcol + 2 * i < p.n ? __bfloat162float(p.bias[gcol + 2 * i]) : 0.f;
          g1 += gcol + 2 * i + 1 < p.n ? __bfloat162float(p.bias[gcol + 2 * i + 1]) : 0.f;
          u0 += ucol + 2 * i < p.n ? __bfloat162float(p.bias[ucol + 2 * i]) : 0.f;
          u1 += ucol + 2 * i + 1 < p.n ? __bfloat162float(p.bias[ucol + 2 * i + 1]) : 0.f;
        }
        const uint32_t s2 = pack_bf16(silu(bf16_round(g0)), silu(bf16_round(g1)));
        pk[i] = as_u32(__hmul2_rn(as_bf2(s2), as_bf2(pack_bf16(u0, u1))));
      }
      emit_packed(o, p, row, tn * (BN / 2) + off + c, cols_out, pk);
    }
  } else if (p.epilogue == kRope) {
    // q/k heads: rotate-half RoPE on the bf16-rounded projection with the reference's
    // rounding points, bf16(bf16(a cos) + bf16(-b sin)) (llama.py:43-45), computed on packed
    // bf16 pairs (a bf16 multiply rounds its exact product once, as the reference's does); v
    // heads: plain. A slice holds whole heads (the host keeps width a multiple of the head size).
    // The fp32 form of the same arithmetic (two roundings and four products per element pair in
    // fp32) had made this epilogue, not the main loop, set the e4m3 q/k/v tile period.
    const int hd = p.rope_hd, half = hd / 2, base = sub * width;
    const int trow = row < p.m ? row : 0;
    // Every head of the tile rotates by the same per-row angles: each 32-column slice of this
    // row's cos / sin is loaded once, packed into bf16 pairs, and used for all the tile's heads.
    const bool any_rot = tn * BN + base + hd <= p.rope_cols;
#pragma unroll 1
    for (int c = 0; c < half; c += 32) {
      uint32_t cp[16], sp[16];  // cos and sin as bf16 pairs (the tables hold bf16-rounded values)
      if (any_rot) {  // 32 consecutive cos / sin of this row: 8 + 8 16-byte loads
        const float4* c4 = reinterpret_cast<const float4*>(p.cos_t + static_cast<int64_t>(trow) * half + c);
        const float4* s4 = reinterpret_cast<const float4*>(p.sin_t + static_cast<int64_t>(trow) * half + c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 cv = c4[i], sv = s4[i];
          cp[2 * i] = pack_bf16(cv.x, cv.y);
          cp[2 * i + 1] = pack_bf16(cv.z, cv.w);
          sp[2 * i] = pack_bf16(sv.x, sv.y);
          sp[2 * i + 1] = pack_bf16(sv.z, sv.w);
        }
      }
#pragma unroll 1
      for (int h0 = 0; h0 < width; h0 += hd) {
        const int hc = tn * BN + base + h0;
        if (hc >= p.n) break;
        uint32_t ra[32], rb[32];
        tmem_ld32(taddr + h0 + c, ra);
        tmem_ld32(taddr + h0 + half + c, rb);
        tmem_wait_ld();
        const bool rot = hc + hd <= p.rope_cols;
        const float wa = FP8 ? pick8(ws, (base + h0 + c) >> 5) : 0.f;
        const float wb = FP8 ? pick8(ws, (base + h0 + half + c) >> 5) : 0.f;
        uint32_t pa[16], pb[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float a0 = __uint_as_float(ra[2 * i]), a1 = __uint_as_float(ra[2 * i + 1]);
          float b0 = __uint_as_float(rb[2 * i]), b1 = __uint_as_float(rb[2 * i + 1]);
          if (FP8) {  // scales by shuffle from the tile's prefetched scales
            a0 *= as * __shfl_sync(0xffffffffu, wa, 2 * i);
            a1 *= as * __shfl_sync(0xffffffffu, wa, 2 * i + 1);
            b0 *= as * __shfl_sync(0xffffffffu, wb, 2 * i);
            b1 *= as * __shfl_sync(0xffffffffu, wb, 2 * i + 1);
          }
          if (p.bias) {
            a0 += __bfloat162float(p.bias[hc + c + 2 * i]);
            a1 += __bfloat162float(p.bias[hc + c + 2 * i + 1]);
            b0 += __bfloat162float(p.bias[hc + half + c + 2 * i]);
            b1 += __bfloat162float(p.bias[hc + half + c + 2 * i + 1]);
          }
          const uint32_t a2 = pack_bf16(a0, a1), b2 = pack_bf16(b0, b1);  // the rounded projection
          if (rot) {
            // bf16(a cos) - bf16(b sin) == bf16(a cos) + bf16(-b sin): negation is exact
            // (the _rn forms: no contraction of a product and a sum into one rounding)
            pa[i] = as_u32(__hsub2_rn(__hmul2_rn(as_bf2(a2), as_bf2(cp[i])), __hmul2_rn(as_bf2(b2), as_bf2(sp[i]))));
            pb[i] = as_u32(__hadd2_rn(__hmul2_rn(as_bf2(b2), as_bf2(cp[i])), __hmul2_rn(as_bf2(a2), as_bf2(sp[i]))));
          } else {
            pa[i] = a2;
            pb[i] = b2;
          }
        }
        emit_packed(o, p, row, hc + c, cols_out, pa);
        emit_packed(o, p, row, hc + half + c, cols_out, pb);
      }
    }
  } else {
    const int col0 = tn * BN + sub * width;
    if (col0 >= p.n) return;
    if (o.tma && p.epilogue == kResidual) {
      residual_tma<FP8>(o, p, taddr, col0, width, as);
      return;
    }
#pragma unroll 1
    for (int c = 0; c < width; c += 32) {
      const int col = col0 + c;
      if (col >= p.n) break;
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      tmem_wait_ld();
      if (FP8) scale_chunk(p, col, as, r);
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float x = __uint_as_float(r[i]);
        if (p.bias && col + i < p.n) x += __bfloat162float(p.bias[col + i]);
        v[i] = x;
      }
      emit<FP8>(o, p, row, col, cols_out, v);
    }
  }
}

template <bool FP8>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                const __grid_constant__ CUtensorMap tc, const __grid_constant__ CUtensorMap tr, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;
  uint8_t* sink = sb + STAGES * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sink + SINK_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // 4 warps x 4 residual-load barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 16);

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    for (int b = 0; b < 16; ++b) mbar_init(&rbar[b], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int k_iters = (p.k * (FP8 ? 1 : 2) + KBYTES - 1) / KBYTES;
  constexpr int KELEM = FP8 ? KBYTES : KBYTES / 2;  // elements of K per stage

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&ta);
      tma_prefetch_desc(&tb);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int tm = t % p.tiles_m, tn = t / p.tiles_m;
        for (int ki = 0; ki < k_iters; ++ki) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            report(p.status, kTimeoutEmpty);
            goto done;
          }
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa + stage * A_BYTES, &ta, &full[stage], ki * KELEM, tm * BM);
          tma_load_2d(sb + stage * B_BYTES, &tb, &full[stage], ki * KELEM, tn * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = FP8 ? idesc_e4m3(BM, BN) : idesc_bf16(BM, BN, false, false);
      int stage = 0, buf = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        if (!mbar_wait(&tempty[buf], acc_phase ^ 1)) {
          report(p.status, kTimeoutEmpty);
          goto done;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int ki = 0; ki < k_iters; ++ki) {
          if (!mbar_wait(&full[stage], phase)) {
            report(p.status, kTimeoutFull);
            goto done;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + stage * A_BYTES), b0 = smem_u32(sb + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t da = desc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t db = desc_sw128(b0 + kk * 32, 16, 1024);
            if (FP8)
              mma_f8_ss(d, da, db, idesc, (ki | kk) != 0);
            else
              mma_f16_ss(d, da, db, idesc, (ki | kk) != 0);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit(&tfull[buf]);
        buf ^= 1;
        if (buf == 0) acc_phase ^= 1;
      }
    }
  } else {
    const int sub = warp & 3;  // TMEM sub-partition this warp may read
    const int r_in = sub * 32 + lane;
    Sink o{p.tma_out != 0, sink + sub * 4 * SLOT_BYTES, rbar + sub * 4, &tc, &tr, 0u, 0u, 0, lane, p.m};
    int buf = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int tm = t % p.tiles_m, tn = t / p.tiles_m;
      epilogue_prefetch(p, tm * BM + r_in, tn);
      float ws[8];
      if (FP8) load_tile_scales(p, tn, lane, ws);
      if (!mbar_wait(&tfull[buf], acc_phase)) {
        report(p.status, kTimeoutMma);
        break;
      }
      tc_fence_after();
      const int row = tm * BM + r_in;
      o.row0 = tm * BM + sub * 32;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(sub * 32) << 16) + buf * BN;
      epilogue_tile<FP8>(p, o, taddr, row, tn, 0, BN, ws);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      buf ^= 1;
      if (buf == 0) acc_phase ^= 1;
    }
    if (lane == 0) bulk_wait_all();  // TMA stores done before the CTA (and its shared memory) ends
  }
done:
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------
// CTA-pair variant (cta_group::2): a cluster of two CTAs on two SMs computes one 256 x 256
// tile. CTA r stages rows [128 r, 128 r + 128) of the tile's A and W slices (32 KB per
// stage, 6 stages); the even CTA issues tcgen05.mma.cta_group::2 (M = 256), which writes
// each CTA's 128 accumulator rows into its own TMEM. Each CTA's TMA loads complete on the
// even CTA's "full" barrier (no multicast); MMA completion is signalled to both CTAs'
// barriers by a multicast commit; the odd CTA's epilogue releases an accumulator buffer on
// the even CTA's barrier through a mapped cluster address. Per SM this halves the W bytes
// staged per FLOP and leaves room for 6 stages.
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * KBYTES, P_B_BYTES = 128 * KBYTES;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + SINK_BYTES + 1024 + 512;

// Stream-K partials: one CTA's 128 x 256 fp32 accumulator of a split-tile segment, stored
// column-major ([col][row]) so a warp's 32 rows of one column are one 128-byte line. Pair q has
// two slots per CTA rank: the first segment of its share (which = 0) and the last (which = 1).
__device__ __forceinline__ float* sk_slot(const Params& p, int q, int rank, int which) {
  return p.sk_part + static_cast<int64_t>((q * 2 + rank) * 2 + which) * BN * 128;
}

// First stream-K iteration of pair q's share.
__device__ __forceinline__ int sk_start(const Params& p, int q, int n_pairs) {
  return static_cast<int>(static_cast<long long>(q) * p.sk_iters / n_pairs);
}

// This warp's 32 rows of its TMEM accumulator -> its slot (``dst`` already offset by the row).
// Not inlined (nor sk_fold): inlined, their 32-value arrays pushed the pair kernel, already at
// 255 registers, into spilling.
__device__ __noinline__ void sk_store_partial(uint32_t taddr, float* dst) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(taddr + c, r);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) __stcg(dst + (c + i) * 128, __uint_as_float(r[i]));
  }
}

// Count this warp's segment of a split tile in; true for the last of the tile's ``n`` segments
// to arrive, which then folds every segment's partial and runs the epilogue. No warp waits for
// another CTA, so the scheme needs no co-residency of the grid. The counter word is (launch
// epoch << 32) | arrivals: a count left by an earlier launch that gave up on a bounded wait is
// restarted, not added to. The CAS loop retries only on a concurrent arrival (at most n times).
__device__ __forceinline__ bool sk_arrive(unsigned long long* cnt, uint32_t epoch, int n, int lane) {
  __threadfence();  // the warp's partial is visible device-wide before it is counted
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    const unsigned long long tag = static_cast<unsigned long long>(epoch) << 32;
    unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(cnt), want;
    for (;;) {
      want = ((old >> 32) == epoch ? old : tag) + 1;
      const unsigned long long seen = atomicCAS(cnt, old, want);
      if (seen == old) break;
      old = seen;
    }
    last = static_cast<int>(want & 0xffffffffull) == n;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) __threadfence();  // the other segments' partials are read after their counts
  return last != 0;
}

// The last arriver of a split tile: the sum of segments qa..qb's partials in pair order (its
// own from TMEM, the others from their slots), the same order whichever segment arrives last,
// so results are deterministic; written back to this warp's TMEM rows for the epilogue.
__device__ __noinline__ void sk_fold(const Params& p, uint32_t taddr, int self, int qa, int qb, int rank,
                                        int tile_start, int n_pairs, int r_in) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t acc[32];
#pragma unroll 1
    for (int q = qa; q <= qb; ++q) {
      uint32_t v[32];
      if (q == self) {
        tmem_ld32(taddr + c, v);
        tmem_wait_ld();
      } else {
        const float* src = sk_slot(p, q, rank, sk_start(p, q, n_pairs) < tile_start ? 1 : 0) + r_in;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__ldcg(src + (c + i) * 128));
      }
#pragma unroll
      for (int i = 0; i < 32; ++i)
        acc[i] = q == qa ? v[i] : __float_as_uint(__uint_as_float(acc[i]) + __uint_as_float(v[i]));
    }
    tmem_st32(taddr + c, acc);
  }
  tmem_wait_st();
}

template <bool FP8>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                     const __grid_constant__ CUtensorMap tbn, const __grid_constant__ CUtensorMap tc,
                     const __grid_constant__ CUtensorMap tr, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + P_STAGES * P_A_BYTES;
  uint8_t* sink = sb + P_STAGES * P_B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sink + SINK_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // 4 warps x 4 residual-load barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 16);

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_rank();  // 0: leader (issues the MMAs), 1: peer
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    for (int b = 0; b < 16; ++b) mbar_init(&rbar[b], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int tiles_m = (p.m + 255) / 256;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int k_iters = (p.k * (FP8 ? 1 : 2) + KBYTES - 1) / KBYTES;
  constexpr int KELEM = FP8 ? KBYTES : KBYTES / 2;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&ta);
      tma_prefetch_desc(&tb);
      if (p.nt_split > 1) tma_prefetch_desc(&tbn);
      int stage = 0;
      uint32_t phase = 0;
      // The operand every wave of tiles touches in full (A for m-fastest order, W for n-fastest)
      // is the one worth keeping in L2; the other streams through.
      const uint64_t keep = l2_evict_last(), pass = l2_evict_normal();
      const uint64_t pol_a = p.order == 0 ? keep : pass, pol_b = p.order == 0 ? pass : keep;
      PairWork work(pair, n_pairs, p, k_iters);
      PairItem w;
      while (work.next(w)) {
        int tm, tn;
        pair_tile(w.t, tiles_m, p.tiles_n, p.order, p.group, tm, tn);
        // Each CTA stages width / 2 rows of W: for SwiGLU its own half of the block's gate or up
        // rows, otherwise its half of the slice's contiguous rows (narrow items use ``tbn``,
        // whose box is width / 2 rows).
        const int bw = w.width / 2;
        const int brow = p.epilogue == kSwiglu ? tn * BN + static_cast<int>(rank) * (BN / 2) + w.sub * bw
                                               : tn * BN + w.sub * w.width + static_cast<int>(rank) * bw;
        const CUtensorMap* mb = w.width == BN ? &tb : &tbn;
        for (int ki = w.kb; ki < w.ke; ++ki) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            report(p.status, kTimeoutEmpty);
            goto done;
          }
          const uint32_t fb = map_shared(smem_u32(&full[stage]), 0);
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * (P_A_BYTES + bw * KBYTES));
          tma_load_2d_pair_hint(sa + stage * P_A_BYTES, &ta, fb, ki * KELEM, tm * 256 + rank * 128, pol_a);
          tma_load_2d_pair_hint(sb + stage * P_B_BYTES, mb, fb, ki * KELEM, brow, pol_b);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && elect_one()) {
      int stage = 0, buf = 0;
      uint32_t phase = 0, acc_phase = 0;
      PairWork work(pair, n_pairs, p, k_iters);
      PairItem w;
      while (work.next(w)) {
        const uint32_t idesc = FP8 ? idesc_e4m3(256, w.width) : idesc_bf16(256, w.width, false, false);
        const int kb = w.kb;
        if (!mbar_wait(&tempty[buf], acc_phase ^ 1)) {
          report(p.status, kTimeoutEmpty);
          goto done;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int ki = kb; ki < w.ke; ++ki) {
          if (!mbar_wait(&full[stage], phase)) {
            report(p.status, kTimeoutFull);
            goto done;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + stage * P_A_BYTES), b0 = smem_u32(sb + stage * P_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t da = desc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t db = desc_sw128(b0 + kk * 32, 16, 1024);
            if (FP8)
              mma_f8_ss_pair(d, da, db, idesc, (ki != kb) || (kk != 0));
            else
              mma_f16_ss_pair(d, da, db, idesc, (ki != kb) || (kk != 0));
          }
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit_pair(&tfull[buf], 0x3);
        buf ^= 1;
        if (buf == 0) acc_phase ^= 1;
      }
    }
  } else {
    const int sub = warp & 3;
    const int r_in = sub * 32 + lane;
    const uint32_t te0 = map_shared(smem_u32(&tempty[0]), 0), te1 = map_shared(smem_u32(&tempty[1]), 0);
    Sink o{p.tma_out != 0, sink + sub * 4 * SLOT_BYTES, rbar + sub * 4, &tc, &tr, 0u, 0u, 0, lane, p.m};
    int buf = 0;
    uint32_t acc_phase = 0;
    const uint32_t epoch = p.sk_iters ? __ldcg(p.sk_ctrl) : 0u;
    PairWork work(pair, n_pairs, p, k_iters);
    PairItem w;
    while (work.next(w)) {
      const int t = w.t, kb = w.kb, ke = w.ke;
      int tm, tn;
      pair_tile(t, tiles_m, p.tiles_n, p.order, p.group, tm, tn);
      const bool split = kb > 0 || ke < k_iters;
      if (!split) epilogue_prefetch(p, tm * 256 + static_cast<int>(rank) * 128 + r_in, tn);
      float ws[8];
      if (FP8 && !split) load_tile_scales(p, tn, lane, ws);
      if (!mbar_wait(&tfull[buf], acc_phase)) {
        report(p.status, kTimeoutMma);
        break;
      }
      tc_fence_after();
      const int row = tm * 256 + static_cast<int>(rank) * 128 + r_in;
      o.row0 = tm * 256 + static_cast<int>(rank) * 128 + sub * 32;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(sub * 32) << 16) + buf * BN;
      bool last = true;  // this warp writes the tile (always, unless the tile is split)
      if (split) {
        // Segments qa..qb of pairs' shares cover this tile; each parks its partial and counts
        // in, and the last to arrive folds them all and writes the tile.
        const int tr = t - p.sk_first, tile_start = tr * k_iters, tile_end = tile_start + k_iters;
        int qa = pair, qb = pair;
        while (sk_start(p, qa, n_pairs) > tile_start) --qa;
        while (qb + 1 < n_pairs && sk_start(p, qb + 1, n_pairs) < tile_end) ++qb;
        const int which = sk_start(p, pair, n_pairs) < tile_start ? 1 : 0;
        sk_store_partial(taddr, sk_slot(p, pair, static_cast<int>(rank), which) + r_in);
        last = sk_arrive(p.sk_cnt + (tr * 2 + static_cast<int>(rank)) * 4 + sub, epoch, qb - qa + 1, lane);
        if (last) {
          if (FP8) load_tile_scales(p, tn, lane, ws);
          sk_fold(p, taddr, pair, qa, qb, static_cast<int>(rank), tile_start, n_pairs, r_in);
        }
      }
      if (last) epilogue_tile<FP8>(p, o, taddr, row, tn, w.sub, w.width, ws);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(buf ? te1 : te0);
      buf ^= 1;
      if (buf == 0) acc_phase ^= 1;
    }
    if (lane == 0) bulk_wait_all();  // TMA stores done before the CTA (and its shared memory) ends
  }
done:
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the pair may still touch its shared memory or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
  if (p.sk_iters && threadIdx.x == 0) {
    // The last CTA out advances the epoch, so the next launch's arrival counts never match this one's.
    __threadfence();
    if (atomicAdd(p.sk_ctrl + 1, 1u) == gridDim.x - 1) {
      p.sk_ctrl[1] = 0;
      __threadfence();
      atomicAdd(p.sk_ctrl, 1u);
    }
  }
}

// Stream-K scratch, one per (device, stream): launches sharing one must be stream-ordered.
// Allocated on first use (cudaMalloc) and kept for the life of the process.
struct Workspace {
  float* part;
  unsigned long long* cnt;
  uint32_t* ctrl;
};

// Partials: two segment slots per (pair, CTA rank), 128 x 256 fp32 each. Counters: one per
// (split tile, CTA rank, epilogue warp), at most 2 x pairs split tiles; then the two control
// words (epoch, CTAs finished).
constexpr size_t sk_part_bytes(int pairs) { return static_cast<size_t>(pairs) * 2 * 2 * BN * 128 * sizeof(float); }
constexpr size_t sk_cnt_bytes(int pairs) {
  return static_cast<size_t>(pairs) * 2 * 2 * 4 * sizeof(unsigned long long) + 2 * sizeof(uint32_t);
}

static Workspace* workspace(cudaStream_t stream, int pairs) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, Workspace> all;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = all.find({dev, stream});
  if (it != all.end()) return &it->second;
  Workspace w{};
  const size_t part_bytes = sk_part_bytes(pairs), cnt_bytes = sk_cnt_bytes(pairs);
  void* a = nullptr;
  void* b = nullptr;
  if (cudaMalloc(&a, part_bytes) != cudaSuccess || cudaMalloc(&b, cnt_bytes) != cudaSuccess ||
      cudaMemset(b, 0, cnt_bytes) != cudaSuccess) {
    if (a) cudaFree(a);
    if (b) cudaFree(b);
    set_error("stream-K workspace allocation of %zu bytes failed", part_bytes + cnt_bytes);
    return nullptr;
  }
  w.part = static_cast<float*>(a);
  w.cnt = static_cast<unsigned long long*>(b);
  w.ctrl = reinterpret_cast<uint32_t*>(w.cnt + static_cast<size_t>(pairs) * 2 * 2 * 4);
  return &(all[{dev, stream}] = w);
}

// Allocation-free stream-K scratch for dan_gemm_bf16_noalloc: one static device array per
// device (zero at module load), laid out like a Workspace for up to kStaticPairs CTA pairs.
constexpr int kStaticPairs = 80;
constexpr size_t kStaticPartBytes = sk_part_bytes(kStaticPairs);
static __device__ __align__(256) unsigned char g_sk_scratch[kStaticPartBytes + sk_cnt_bytes(kStaticPairs)];

// The static scratch of the current device as a Workspace (its address looked up once per
// device with cudaGetSymbolAddress); nullptr with the error text set if it is unavailable.
static const Workspace* static_workspace() {
  static std::mutex mu;
  static std::map<int, Workspace> all;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = all.find(dev);
  if (it != all.end()) return &it->second;
  void* base = nullptr;
  if (cudaGetSymbolAddress(&base, g_sk_scratch) != cudaSuccess) {
    set_error("cudaGetSymbolAddress of the static stream-K scratch failed");
    return nullptr;
  }
  Workspace w{};
  w.part = static_cast<float*>(base);
  w.cnt = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(base) + kStaticPartBytes);
  w.ctrl = reinterpret_cast<uint32_t*>(w.cnt + static_cast<size_t>(kStaticPairs) * 2 * 2 * 4);
  return &(all[dev] = w);
}

// ``fixed``: use this stream-K workspace (sized for kStaticPairs) instead of allocating one.
template <bool FP8>
int launch(const void* a, int64_t lda, const void* w, int64_t ldw, Params p, cudaStream_t stream,
           const Workspace* fixed = nullptr) {
  const int esize = FP8 ? 1 : 2;
  DAN_REQUIRE(p.m > 0 && p.n > 0 && p.k > 0, "gemm: empty problem m=%d n=%d k=%d", p.m, p.n, p.k);
  DAN_REQUIRE((p.k * esize) % 16 == 0, "gemm: k=%d must make 16-byte rows", p.k);
  DAN_REQUIRE((lda * esize) % 16 == 0 && (ldw * esize) % 16 == 0, "gemm: lda/ldw must be 16-byte multiples");
  DAN_REQUIRE(lda >= p.k && ldw >= p.k, "gemm: leading dimensions smaller than k");
  DAN_REQUIRE(p.epilogue >= 0 && p.epilogue <= 3, "gemm: unknown epilogue %d", p.epilogue);
  DAN_REQUIRE(p.epilogue != kRope || ((p.rope_hd == 64 || p.rope_hd == 128 || p.rope_hd == 256) &&
                                      p.rope_cols % p.rope_hd == 0 && p.n % p.rope_hd == 0 && p.cos_t && p.sin_t),
              "gemm: rope epilogue needs head size 64/128/256 dividing n and rope_cols, and cos/sin tables");
  DAN_REQUIRE(p.epilogue != kSwiglu || p.n % BN == 0, "gemm: swiglu needs n %% 256 == 0 (got %d)", p.n);
  DAN_REQUIRE(p.epilogue != kResidual || p.resid != nullptr, "gemm: residual epilogue without a residual");
  DAN_REQUIRE(!FP8 || (p.a_scale && p.w_scale), "gemm: e4m3 needs a_scale and w_scale");
  CUtensorMap ta, tb;
  const CUtensorMapDataType dt = FP8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t kbox = KBYTES / esize;
  {
    uint64_t dims[2] = {static_cast<uint64_t>(p.k), static_cast<uint64_t>(p.m)};
    uint64_t strides[1] = {static_cast<uint64_t>(lda) * esize};
    uint32_t box[2] = {kbox, BM};
    int rc = make_tmap(&ta, a, dt, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    uint64_t dims[2] = {static_cast<uint64_t>(p.k), static_cast<uint64_t>(p.n)};
    uint64_t strides[1] = {static_cast<uint64_t>(ldw) * esize};
    uint32_t box[2] = {kbox, BN};
    int rc = make_tmap(&tb, w, dt, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  // Output (and residual) maps for the TMA-store epilogue: 32 x 32 bf16 boxes, no swizzle.
  CUtensorMap tc{}, tr{};
  {
    const int cols_out = p.epilogue == kSwiglu ? p.n / 2 : p.n;
    const auto aligned = [](const void* q, int64_t ld) {
      return (reinterpret_cast<uintptr_t>(q) & 15) == 0 && (ld * 2) % 16 == 0;
    };
    p.tma_out = aligned(p.c, p.ldc) && (p.epilogue != kResidual || aligned(p.resid, p.ldr));
    if (p.tma_out) {
      uint64_t dims[2] = {static_cast<uint64_t>(cols_out), static_cast<uint64_t>(p.m)};
      uint64_t strides[1] = {static_cast<uint64_t>(p.ldc) * 2};
      uint32_t box[2] = {32, 32};
      int rc = make_tmap(&tc, p.c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
      tr = tc;
      if (p.epilogue == kResidual) {
        uint64_t rdims[2] = {static_cast<uint64_t>(p.n), static_cast<uint64_t>(p.m)};
        uint64_t rstrides[1] = {static_cast<uint64_t>(p.ldr) * 2};
        rc = make_tmap(&tr, p.resid, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rdims, rstrides, box,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
      }
    }
  }
  p.tiles_m = (p.m + BM - 1) / BM;
  p.tiles_n = (p.n + BN - 1) / BN;
  if (p.m >= 256) {  // CTA pairs: 256 x 256 tiles, each CTA stages 128 rows of A and of W
    CUtensorMap tb2;
    uint64_t dims[2] = {static_cast<uint64_t>(p.k), static_cast<uint64_t>(p.n)};
    uint64_t strides[1] = {static_cast<uint64_t>(ldw) * esize};
    uint32_t box[2] = {kbox, 128};
    int rc = make_tmap(&tb2, w, dt, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const int tiles = ((p.m + 255) / 256) * p.tiles_n;
    // Rasterization: the smaller operand is the stationary one (every wave of a group re-reads
    // its slice, held in L2 with an evict_last policy) and tiles are grouped so that the
    // stationary slice of a group is at most kGroupBytes (data read by SMs of both dies only
    // gets about half of the 126 MB L2).
    p.order = static_cast<int64_t>(p.m) <= p.n ? 0 : 1;
    const int gdim = p.order == 0 ? (p.m + 255) / 256 : p.tiles_n;
    const int64_t grp = kGroupBytes / (256LL * p.k * esize);
    p.group = grp < 1 ? 1 : (grp < gdim ? static_cast<int>(grp) : gdim);
    const int max_pairs = sm_count() / 2;
    int pairs = tiles < max_pairs ? tiles : max_pairs;
    // Stream-K when whole tiles would leave the last wave less than 95% busy and a tile is at
    // least 128 K iterations deep: the last (tiles % P) + P tiles (all of them if there are
    // fewer than P) are split evenly by K iteration over all P pairs. Shallower tiles do not
    // repay the partial-tile traffic and the reduction in the owning pair's epilogue.
    p.sk_first = tiles;
    p.sk_iters = 0;
    {
      const int k_iters = (p.k * esize + KBYTES - 1) / KBYTES;
      const int waves = (tiles + max_pairs - 1) / max_pairs;
      const bool ragged = static_cast<int64_t>(tiles) * 100 < static_cast<int64_t>(waves) * max_pairs * 95;
      const int first = tiles <= max_pairs ? 0 : (tiles / max_pairs - 1) * max_pairs;
      const int64_t iters = static_cast<int64_t>(tiles - first) * k_iters;
      if (ragged && k_iters >= 128 && iters >= 8LL * max_pairs) {
        const Workspace* ws = fixed;
        if (ws && max_pairs > kStaticPairs)
          return fail(-22, "gemm: %d CTA pairs exceed the static stream-K scratch (%d pairs)", max_pairs,
                      kStaticPairs);
        if (!ws) ws = workspace(stream, max_pairs);
        if (!ws) return fail(2, "gemm: %s", last_error());
        p.sk_first = first;
        p.sk_iters = static_cast<int>(iters);
        p.sk_part = ws->part;
        p.sk_cnt = ws->cnt;
        p.sk_ctrl = ws->ctrl;
        pairs = max_pairs;
      }
    }
    // Narrow tail: without stream-K, the tiles of a ragged last wave each run as s items of
    // 256 / s columns (s = 2, 4 or 8, as many as the pairs can take at once), so that wave
    // ends sooner instead of leaving most pairs idle. A narrow item still streams the tile's
    // whole A slice, so it costs more than 1 / s of a tile, but several times less than one.
    // SwiGLU items keep >= 32 gate and up columns; RoPE items keep whole heads.
    p.nt_first = p.sk_first;
    p.nt_split = 1;
    CUtensorMap tbn = tb2;
    if (p.sk_iters == 0) {
      const int rem = tiles % max_pairs;
      int s_max = 8;
      if (p.epilogue == kSwiglu) s_max = 4;
      if (p.epilogue == kRope) s_max = BN / p.rope_hd;
      int s = 1;
      while (2 * s <= s_max && rem * 2 * s <= max_pairs) s *= 2;
      if (rem > 0 && s > 1) {
        p.nt_first = tiles - rem;
        p.nt_split = s;
        uint64_t dims[2] = {static_cast<uint64_t>(p.k), static_cast<uint64_t>(p.n)};
        uint64_t strides[1] = {static_cast<uint64_t>(ldw) * esize};
        uint32_t box[2] = {kbox, static_cast<uint32_t>(BN / s / 2)};
        int rc = make_tmap(&tbn, w, dt, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        const int items = p.nt_first + rem * s;
        pairs = items < max_pairs ? items : max_pairs;
      }
    }
    static std::atomic<uint64_t> pconf{0};
    DAN_CUDA(smem_limit_once(gemm_pair_kernel<FP8>, P_SMEM_BYTES, pconf));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    DAN_CUDA(cudaLaunchKernelEx(&cfg, gemm_pair_kernel<FP8>, ta, tb2, tbn, tc, tr, p));
    return 0;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  constexpr int smem_bytes = SMEM_BYTES_BASE + SINK_BYTES;
  static std::atomic<uint64_t> configured{0};
  DAN_CUDA(smem_limit_once(gemm_kernel<FP8>, smem_bytes, configured));
  gemm_kernel<FP8><<<grid, THREADS, smem_bytes, stream>>>(ta, tb, tc, tr, p);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

}  // namespace gemm
}  // namespace dan

using namespace dan;

DAN_API int dan_gemm_bf16_rope(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
                               const void* resid, int64_t ldr, const void* bias, int m, int n, int k, int epilogue,
                               int rope_cols, int rope_hd, const float* cos_t, const float* sin_t, int32_t* status,
                               void* stream);
DAN_API int dan_gemm_e4m3_rope(const void* a, int64_t lda, const float* a_scale, const void* w, int64_t ldw,
                               const float* w_scale, void* c, int64_t ldc, const void* resid, int64_t ldr,
                               const void* bias, int m, int n, int k, int epilogue, int rope_cols, int rope_hd,
                               const float* cos_t, const float* sin_t, int32_t* status, void* stream);

DAN_API int dan_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
                          const void* resid, int64_t ldr, const void* bias, int m, int n, int k, int epilogue,
                          int32_t* status, void* stream) {
  return dan_gemm_bf16_rope(a, lda, w, ldw, c, ldc, resid, ldr, bias, m, n, k, epilogue, 0, 0, nullptr, nullptr,
                            status, stream);
}

DAN_API int dan_gemm_bf16_rope(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
                               const void* resid, int64_t ldr, const void* bias, int m, int n, int k, int epilogue,
                               int rope_cols, int rope_hd, const float* cos_t, const float* sin_t, int32_t* status,
                               void* stream) {
  gemm::Params p{};
  p.rope_cols = rope_cols;
  p.rope_hd = rope_hd;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  p.resid = static_cast<const __nv_bfloat16*>(resid);
  p.ldr = ldr;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.m = m;
  p.n = n;
  p.k = k;
  p.epilogue = epilogue;
  p.status = status;
  return gemm::launch<false>(a, lda, w, ldw, p, static_cast<cudaStream_t>(stream));
}

DAN_API int dan_gemm_bf16_noalloc(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
                                  const void* resid, int64_t ldr, const void* bias, int m, int n, int k,
                                  int epilogue, int32_t* status, void* stream) {
  const gemm::Workspace* ws = gemm::static_workspace();
  if (!ws) return fail(2, "gemm: %s", last_error());
  gemm::Params p{};
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  p.resid = static_cast<const __nv_bfloat16*>(resid);
  p.ldr = ldr;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.m = m;
  p.n = n;
  p.k = k;
  p.epilogue = epilogue;
  p.status = status;
  return gemm::launch<false>(a, lda, w, ldw, p, static_cast<cudaStream_t>(stream), ws);
}

DAN_API int dan_gemm_e4m3(const void* a, int64_t lda, const float* a_scale, const void* w, int64_t ldw,
                          const float* w_scale, void* c, int64_t ldc, const void* resid, int64_t ldr,
                          const void* bias, int m, int n, int k, int epilogue, int32_t* status, void* stream) {
  return dan_gemm_e4m3_rope(a, lda, a_scale, w, ldw, w_scale, c, ldc, resid, ldr, bias, m, n, k, epilogue, 0, 0,
                            nullptr, nullptr, status, stream);
}

DAN_API int dan_gemm_e4m3_rope(const void* a, int64_t lda, const float* a_scale, const void* w, int64_t ldw,
                               const float* w_scale, void* c, int64_t ldc, const void* resid, int64_t ldr,
                               const void* bias, int m, int n, int k, int epilogue, int rope_cols, int rope_hd,
                               const float* cos_t, const float* sin_t, int32_t* status, void* stream) {
  gemm::Params p{};
  p.rope_cols = rope_cols;
  p.rope_hd = rope_hd;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  p.resid = static_cast<const __nv_bfloat16*>(resid);
  p.ldr = ldr;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.a_scale = a_scale;
  p.w_scale = w_scale;
  p.m = m;
  p.n = n;
  p.k = k;
  p.epilogue = epilogue;
  p.status = status;
  return gemm::launch<true>(a, lda, w, ldw, p, static_cast<cudaStream_t>(stream));
}
