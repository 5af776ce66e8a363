// Tree-masked attention for packed prefill reads, one kernel for the whole batch.
//
// Replaces the reference's three flash varlen calls + log-sum-exp merge + row
// gathers (dan/attention.py:210-241; dense semantics 244-270). A query may see
// a key when the key comes first and is trunk (cached past included) or in the
// query's own branch (attention.py:6-13).
//
// Virtual key index space of a segment: [0, P) cached past keys (pool pages of
// 128 tokens), [P, Ppad) padding (never visible, Ppad = P rounded up to 128),
// then the segment's new tokens in packed order: trunk [Ppad, split), branches
// [split, Ppad + len). A query row with virtual index qv whose own run starts
// at ``own`` sees key v iff
//     v <= qv  and  (v < split or v >= own)  and  (v < P or v >= Ppad).
// Trunk rows have qv < split, so the middle clause is true for them; branch
// rows see every trunk key and their own branch causally.
//
// Work unit: one 128-row query tile of one segment x one query head (CTA).
// The host lists, per tile, the key blocks it needs: blocks [0, nblk_a) over
// past + trunk, then [blk_b0, blk_b1) over the tile's own branch region;
// every other block is fully masked and skipped. A block that is fully
// visible to every row of the tile skips the mask arithmetic.
//
// Pipeline of the single-head kernel (warp-specialised, 320 threads):
//   warp 0   TMA producer: Q once, then K_j / V_j into an NS-deep ring
//            (packed rows of the current batch, or pool pages for past keys);
//   warp 1   MMA issuer: S_j = Q K_j^T into TMEM buffer j&1 (SS MMA); after the
//            softmax has written P_j (bf16) over S_j, O += P_j V_j with P read
//            from TMEM (TS MMA) and V as an MN-major shared-memory operand;
//   warps 2-9 softmax, 16 rows each with two threads per row (16x32bx2 TMEM
//            shape: one thread per 64 keys of a block and half of O's columns):
//            online softmax in the log2 domain; O is rescaled lazily, only when a
//            row max grows by more than 2^8 (exact: the same stale max is used for
//            P and for l); then the epilogue O / l -> bf16. With one thread per row
//            (four softmax warps) it ran 686 TFLOP/s at 16 / 4 heads x 256 on a
//            configuration-4 batch, with two 825.
// TMEM: S0 [0,128), S1 [128,256), O [256, 256 + D).
#include "common.cuh"

namespace dan {
namespace attn {

constexpr int BM = 128, BN = 128;
constexpr int THREADS = 320;  // single-head kernel: TMA warp, MMA warp, 8 softmax warps
constexpr int CHUNK = 128 * 128;  // bytes of one 64-column x 128-row bf16 box

struct Tile {
  int row0, nrows, seg_start, past, ppad, split, nblk_a, blk_b0, blk_b1, page0, q0v, pad;
};

struct Params {
  __nv_bfloat16* out;
  int64_t out_row, out_head;
  const int* tiles;
  const int* row_own;
  const int* pages;
  int n_rows, n_heads, n_kv_heads;
  float scale_log2;
  int32_t* status;
  const int* sched;  // optional: [ctas + 1] CSR offsets, then the item ids of each CTA
  int sched_ctas;
};

// The k-th work item of this CTA, or -1: from the host's LPT schedule when given,
// else round-robin over the LPT-sorted items.
__device__ __forceinline__ int item_at(const Params& p, int k, int n_items) {
  if (p.sched) {
    const int b = p.sched[blockIdx.x] + k;
    return b < p.sched[blockIdx.x + 1] ? p.sched[p.sched_ctas + 1 + b] : -1;
  }
  const int w = blockIdx.x + k * gridDim.x;
  return w < n_items ? w : -1;
}

template <int D>
struct Cfg {
  static constexpr int NS = D <= 64 ? 3 : (D <= 128 ? 2 : 1);
  static constexpr int CHUNKS = D / 64;
  static constexpr int Q_BYTES = CHUNKS * CHUNK;
  static constexpr int KV_BYTES = CHUNKS * CHUNK;
  // Output staging: per softmax warp two 1 KB slots (16 rows x 32 bf16 columns, one per
  // column half, 64-byte swizzle) sent by TMA store.
  static constexpr int SLOT_BYTES = 16 * 64;
  static constexpr int SINK_BYTES = 8 * 2 * SLOT_BYTES;
  // At least 120 KB so two CTAs never share an SM: each allocates all 512 TMEM columns.
  static constexpr int SMEM_USED = Q_BYTES + 2 * NS * KV_BYTES + SINK_BYTES + 1024 + 512;
  static constexpr int SMEM = SMEM_USED < 120 * 1024 ? 120 * 1024 : SMEM_USED;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// bits [lo, hi) of a 32-bit word (arguments relative to the word's first column)
__device__ __forceinline__ uint32_t span_bits(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 32);
  if (hi <= lo) return 0u;
  const uint32_t upto = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
  return upto & ~((1u << lo) - 1u);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic) and the three-input max: the softmax warps are
// issue-bound, and these halve the instructions per score of the max, scale and sum steps.
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of floats on the FMA pipe (packed f32x2), sharing the exponentials with the
// MUFU unit, which limits the softmax otherwise (one warp's 4096 exponentials per block are
// 1024 MUFU cycles on its SM sub-partition). Cody-Waite range reduction x = n + f with
// n = round(x) taken from a magic-constant add (1.5 * 2^23) and f in [-1/2, 1/2]; 2^f by a
// degree-3 polynomial (coefficients fitted for this kernel by weighted least squares toward
// minimax: max relative error 7.7e-5, far below the bf16 rounding P takes next); 2^n added
// into the exponent bits. For finite x <= 8; x below -125 gives 2^-125, not 0, so only fully
// visible chunks (no -inf scores) use it.
__device__ __forceinline__ void exp2_pair_fma(uint64_t x2, float& ra, float& rb) {
  float xa, xb;
  f2_split(x2, xa, xb);
  const uint64_t xc = f2(fmaxf(xa, -125.f), fmaxf(xb, -125.f));
  const uint64_t t = fadd2(xc, f2(12582912.f, 12582912.f));
  const uint64_t n = fadd2(t, f2(-12582912.f, -12582912.f));
  const uint64_t f = ffma2(n, f2(-1.f, -1.f), xc);
  uint64_t q = ffma2(f2(0.05518098f, 0.05518098f), f, f2(0.24263459f, 0.24263459f));
  q = ffma2(q, f, f2(0.69326133f, 0.69326133f));
  q = ffma2(q, f, f2(0.99992621f, 0.99992621f));
  float qa, qb, ta, tb;
  f2_split(q, qa, qb);
  f2_split(t, ta, tb);
  ra = __int_as_float(__float_as_int(qa) + (__float_as_int(ta) << 23));
  rb = __int_as_float(__float_as_int(qb) + (__float_as_int(tb) << 23));
}

// One score pair in EXP_EMU_EVERY of a fully visible chunk takes exp2_pair_fma. With four
// softmax warps per SM sub-partition the MUFU unit is rarely the limit and the emulation's
// extra instructions cost more than they free (configuration-2 batch, TFLOP/s: 1 in 2 730,
// 1 in 4 775, 1 in 8 783, 1 in 16 792, none 782-790; with one softmax thread per row it had
// been none 535, 1 in 4 551, 1 in 2 532). Writing an item's output after the next item's
// first unit instead of before it measured 1% slower.
constexpr int EXP_EMU_EVERY = 16;

// Masked scores become -inf in place (partially visible chunks then take the packed path:
// exp2(-inf) = 0 and -inf never wins a max).
__device__ __forceinline__ void mask_chunk(uint32_t (&s)[32], uint32_t mw) {
#pragma unroll
  for (int i = 0; i < 32; ++i) s[i] = ((mw >> i) & 1u) ? s[i] : 0xff800000u;
}

// Row max over 32 scores (already masked, or all visible).
__device__ __forceinline__ void chunk_max(const uint32_t (&s)[32], float& mx) {
  float a = fmax3(__uint_as_float(s[0]), __uint_as_float(s[1]), __uint_as_float(s[2]));
  float b = fmax3(__uint_as_float(s[3]), __uint_as_float(s[4]), __uint_as_float(s[5]));
#pragma unroll
  for (int i = 6; i + 3 < 32; i += 4) {
    a = fmax3(a, __uint_as_float(s[i]), __uint_as_float(s[i + 1]));
    b = fmax3(b, __uint_as_float(s[i + 2]), __uint_as_float(s[i + 3]));
  }
  mx = fmax3(mx, fmax3(a, b, __uint_as_float(s[30])), __uint_as_float(s[31]));
}

// P = exp2(s * scale_log2 - m) for 32 scores (masked ones are -inf and give 0) as 16 bf16
// pairs; with ``emu`` (a fully visible chunk) every EXP_EMU_EVERY-th pair on the FMA pipe.
template <bool EMU>
__device__ __forceinline__ void chunk_exp(const uint32_t (&s)[32], float sl2, float mu, float& sum,
                                          uint32_t (&pk)[16]) {
  const uint64_t scale = f2(sl2, sl2), shift = f2(-mu, -mu);
  uint64_t acc = f2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint64_t x2 = ffma2(f2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), scale, shift);
    float a, b;
    if (EMU && i % EXP_EMU_EVERY == EXP_EMU_EVERY - 1) {
      exp2_pair_fma(x2, a, b);
    } else {
      float xa, xb;
      f2_split(x2, xa, xb);
      a = fast_exp2(xa);
      b = fast_exp2(xb);
    }
    acc = fadd2(acc, f2(a, b));
    pk[i] = pack_bf16(a, b);
  }
  float s0, s1;
  f2_split(acc, s0, s1);
  sum += s0 + s1;
}

// Warp-uniform forms (``cls``: 0 no lane sees a key of the chunk, 1 mixed, 2 every lane sees
// every key).
__device__ __forceinline__ void chunk_prep_u(uint32_t (&s)[32], uint32_t mw, uint32_t cls, float& mx) {
  if (cls == 0u) return;
  if (cls == 1u) mask_chunk(s, mw);
  chunk_max(s, mx);
}
__device__ __forceinline__ void chunk_p_u(const uint32_t (&s)[32], uint32_t cls, float sl2, float mu, float& sum,
                                          uint32_t (&pk)[16]) {
  if (cls == 0u) {
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = 0u;
  } else if (cls == 2u) {
    chunk_exp<true>(s, sl2, mu, sum, pk);
  } else {
    chunk_exp<false>(s, sl2, mu, sum, pk);
  }
}

template <int D>
__global__ void __launch_bounds__(THREADS, 1)
    tree_attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tpk,
                          const __grid_constant__ CUtensorMap tpv, const __grid_constant__ CUtensorMap to,
                          Params p) {
  using C = Cfg<D>;
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sk = sq + C::Q_BYTES;
  uint8_t* sv = sk + NS * C::KV_BYTES;
  uint8_t* sink = sv + NS * C::KV_BYTES;  // 1024-byte aligned: Q and K/V stages are multiples of 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sink + C::SINK_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + NS;
  uint64_t* k_empty = v_full + NS;
  uint64_t* v_empty = k_empty + NS;
  uint64_t* s_full = v_empty + NS;   // [2]
  uint64_t* p_full = s_full + 2;     // [2]
  uint64_t* pv_done = p_full + 2;    // [2] indexed by block parity
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);

  const int head = blockIdx.x;
  const int kvh = head / (p.n_heads / p.n_kv_heads);
  const Tile tile = reinterpret_cast<const Tile*>(p.tiles)[blockIdx.y];
  const int nblk = tile.nblk_a + (tile.blk_b1 - tile.blk_b0);
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);
      mbar_init(&pv_done[b], 1);
    }
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
  const uint32_t tmem_o = tmem + 256;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < C::CHUNKS; ++c) tma_load_3d(sq + c * CHUNK, &tq, q_full, c * 64, head, tile.row0);
      for (int j = 0; j < nblk; ++j) {
        const int stage = j % NS;
        const uint32_t ph = (j / NS) & 1;
        const int b = j < tile.nblk_a ? j : tile.blk_b0 + (j - tile.nblk_a);
        const int kb = b * BN;
        const bool pool = kb < tile.ppad;
        const int row = pool ? p.pages[tile.page0 + b] * BN : tile.seg_start + (kb - tile.ppad);
        const CUtensorMap* mk = pool ? &tpk : &tk;
        const CUtensorMap* mv = pool ? &tpv : &tv;
        if (!mbar_wait(&k_empty[stage], ph ^ 1)) {
          report(p.status, kTimeoutEmpty);
          break;
        }
        mbar_expect_tx(&k_full[stage], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c)
          tma_load_3d(sk + stage * C::KV_BYTES + c * CHUNK, mk, &k_full[stage], c * 64, kvh, row);
        if (!mbar_wait(&v_empty[stage], ph ^ 1)) {
          report(p.status, kTimeoutEmpty);
          break;
        }
        mbar_expect_tx(&v_full[stage], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c)
          tma_load_3d(sv + stage * C::KV_BYTES + c * CHUNK, mv, &v_full[stage], c * 64, kvh, row);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(BM, D, false, true);
      bool ok = mbar_wait(q_full, 0);
      if (!ok) report(p.status, kTimeoutFull);
      tc_fence_after();
      const uint32_t q0 = smem_u32(sq);
      auto issue_pv = [&](int i) -> bool {
        const int st = i % NS;
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1)) {
          report(p.status, kTimeoutSoftmax);
          return false;
        }
        if (!mbar_wait(&v_full[st], (i / NS) & 1)) {
          report(p.status, kTimeoutFull);
          return false;
        }
        tc_fence_after();
        const uint32_t v0 = smem_u32(sv + st * C::KV_BYTES);
        const uint32_t pa = tmem + (i & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t db = desc_sw128(v0 + kk * 2048, CHUNK, 1024);
          mma_f16_ts(tmem_o, pa + kk * 8, db, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&v_empty[st]);
        mma_commit(&pv_done[i & 1]);
        return true;
      };
      for (int j = 0; ok && j < nblk; ++j) {
        const int stage = j % NS;
        if (j >= 2 && !mbar_wait(&pv_done[j & 1], ((j - 2) >> 1) & 1)) {
          report(p.status, kTimeoutMma);
          break;
        }
        if (!mbar_wait(&k_full[stage], (j / NS) & 1)) {
          report(p.status, kTimeoutFull);
          break;
        }
        tc_fence_after();
        const uint32_t k0 = smem_u32(sk + stage * C::KV_BYTES);
        const uint32_t sd = tmem + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_f16_ss(sd, desc_sw128(q0 + off, 16, 1024), desc_sw128(k0 + off, 16, 1024), idesc_qk, kk > 0);
        }
        mma_commit(&s_full[j & 1]);
        mma_commit(&k_empty[stage]);
        if (j >= 1 && !issue_pv(j - 1)) break;
        if (j == nblk - 1) issue_pv(j);
      }
    }
  } else {
    // softmax + epilogue: warp w (2..9) covers 16 rows of its TMEM lane quarter (w % 4), two
    // threads per row (the 16x32bx2 access shape): thread t < 16 takes row t and keys [0, 64)
    // of each block (the first half of O's columns), thread t + 16 keys [64, 128) (the second
    // half); the halves of a row share their maximum by one shuffle.
    const int sidx = warp - 2;       // 0..7
    const int sub = warp & 3;        // TMEM lane quarter
    const int half = lane >> 4;
    const int r0 = sub * 32 + (sidx >> 2) * 16;  // first tile row of this warp
    const int r_in = r0 + (lane & 15);
    const int row = tile.row0 + r_in;
    const bool valid = r_in < tile.nrows;
    const int qv = tile.q0v + r_in;
    const int own = valid ? tile.ppad + (p.row_own[row] - tile.seg_start) : tile.ppad;
    const int e_past = min(tile.past, qv + 1), e_trunk = min(tile.split, qv + 1);
    const uint32_t lane_base = static_cast<uint32_t>(r0) << 16;
    const uint32_t o_addr = tmem_o + lane_base;
    const float sl2 = p.scale_log2;
    uint8_t* wslots = sink + sidx * 2 * C::SLOT_BYTES;  // per key half: 16 rows x 32 columns
    uint8_t* slot = wslots + half * C::SLOT_BYTES;
    float m = -INFINITY, l = 0.f;  // m in log2 units (scaled); l over this thread's keys
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j < tile.nblk_a ? j : tile.blk_b0 + (j - tile.nblk_a);
      const int kb = b * BN;
      const bool full = (kb + BN <= tile.past) ||
                        (kb >= tile.ppad && kb + BN <= tile.split && kb + BN - 1 <= tile.q0v);
      uint32_t mw[2], cls[2];  // this thread's two 32-key chunks: [kb + 64 half + 32 c, + 32)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int base = kb + 64 * half + 32 * c;
        mw[c] = full ? 0xffffffffu
                     : (span_bits(-base, e_past - base) | span_bits(tile.ppad - base, e_trunk - base) |
                        span_bits(own - base, qv + 1 - base));
        cls[c] = full ? 2u
                      : (__all_sync(0xffffffffu, mw[c] == 0xffffffffu)
                             ? 2u
                             : (__any_sync(0xffffffffu, mw[c] != 0u) ? 1u : 0u));
      }
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1)) {
        report(p.status, kTimeoutMma);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = tmem + lane_base + (j & 1) * 128;
      uint32_t x[32], y[32];
      tmem_ld16x2_x32<64>(sa, x);
      tmem_ld16x2_x32<64>(sa + 32, y);
      tmem_wait_ld_regs(x);
      tmem_wait_ld_regs(y);
      float mx = -INFINITY;
      chunk_prep_u(x, mw[0], cls[0], mx);
      chunk_prep_u(y, mw[1], cls[1], mx);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m, mx * sl2);
      bool rescale = false;
      float alpha = 1.f;
      if (m_new != -INFINITY) {
        if (m == -INFINITY) {
          m = m_new;  // nothing accumulated yet for this row: O row and l are zero
        } else if (m_new > m + 8.f) {
          alpha = fast_exp2(m - m_new);
          m = m_new;
          rescale = true;
        }
      }
      const float mu = m == -INFINITY ? 0.f : m;
      float sum = 0.f;
      {
        uint32_t pk[16];
        chunk_p_u(x, cls[0], sl2, mu, sum, pk);
        tmem_st16x2_x16<32>(sa, pk);  // keys [64 half, +32) -> P columns [32 half, +16)
        chunk_p_u(y, cls[1], sl2, mu, sum, pk);
        tmem_st16x2_x16<32>(sa + 16, pk);
      }
      l = l * alpha + sum;
      if (__any_sync(0xffffffffu, rescale) && j > 0) {
        // O holds sum_{i<j} P_i V_i once PV_{j-1} completes; scale this thread's half of it.
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
          report(p.status, kTimeoutMma);
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 2; c += 32) {
          uint32_t o[32];
          tmem_ld16x2_x32<D / 2>(o_addr + c, o);
          tmem_wait_ld_regs(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16x2_x32<D / 2>(o_addr + c, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
    }
    if (ok && nblk > 0) {
      const int last = nblk - 1;
      if (!mbar_wait(&pv_done[last & 1], (last >> 1) & 1)) {
        report(p.status, kTimeoutMma);
      } else {
        tc_fence_after();
        const float lt = l + __shfl_xor_sync(0xffffffffu, l, 16);
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        // Whole 16-row slabs leave through the warp's shared-memory slots by TMA store (as in the
        // paired kernel); a segment's ragged last rows are stored per row.
        const bool slab = r0 + 16 <= tile.nrows;
        __nv_bfloat16* dst = p.out + static_cast<int64_t>(row) * p.out_row + static_cast<int64_t>(head) * p.out_head;
#pragma unroll 1
        for (int c = 0; c < D / 2; c += 32) {
          uint32_t o[32];
          tmem_ld16x2_x32<D / 2>(o_addr + c, o);
          tmem_wait_ld_regs(o);
          uint32_t pkd[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pkd[i] = pack_bf16(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
          if (slab) {
            if (lane == 0) bulk_wait_read<0>();  // the previous stores from these slots have read them
            __syncwarp();
            const int r = lane & 15;  // 64-byte swizzle: unit u of row r at u ^ ((r >> 1) & 3)
            uint4* d4 = reinterpret_cast<uint4*>(slot + r * 64);
            const int sw = (r >> 1) & 3;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              d4[i ^ sw] = make_uint4(pkd[4 * i], pkd[4 * i + 1], pkd[4 * i + 2], pkd[4 * i + 3]);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&to, wslots, c, head, tile.row0 + r0);
              tma_store_3d(&to, wslots + C::SLOT_BYTES, D / 2 + c, head, tile.row0 + r0);
              bulk_commit();
            }
            __syncwarp();
          } else if (valid) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + half * (D / 2) + c);
#pragma unroll
            for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pkd[4 * i], pkd[4 * i + 1], pkd[4 * i + 2], pkd[4 * i + 3]);
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // output stores done before the CTA's shared memory goes away
    tc_fence_before();
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tpk,
           const CUtensorMap& tpv, const CUtensorMap& to, const Params& p, int n_tiles, cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  DAN_CUDA(smem_limit_once(tree_attention_kernel<D>, Cfg<D>::SMEM, configured));
  dim3 grid(p.n_heads, n_tiles);
  tree_attention_kernel<D><<<grid, THREADS, Cfg<D>::SMEM, stream>>>(tq, tk, tv, tpk, tpv, to, p);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

// ---------------------------------------------------------------------------------
// Paired-head persistent variant. A work item is one 128-row query tile x two query
// heads that share a KV head (GQA): both heads have the same key blocks and masks, so
// each K/V tile is loaded once for 2 x 128 query rows. One CTA per SM walks the
// LPT-ordered items (tile-major, so CTAs running at the same time share K/V in L2) with
// barrier phases carried across items.
// Each 128-key block is consumed as two 64-key units, and each head has two 64-column S
// buffers in TMEM (unit k in buffer k & 1), so the tensor core computes S_h(k + 2) while
// the softmax warps of head h are still on unit k + 1: a head's softmax never waits for
// its own PV and QK products. MMA issue order per item of n units:
//   QK0(0) QK0(1) QK1(0) QK1(1) | PV0(k) QK0(k+2) PV1(k) QK1(k+2) | ... PV0(n-1) PV1(n-1)
// (the next item's first QK products run while the softmax warps store this item's output).
// QK_h(k+2) overwrites the buffer that held P_h(k) only after PV_h(k), issued before it
// by the same thread, has read it (tcgen05 MMAs of one thread run in issue order). A
// commit arrives only after every earlier MMA of the issuing thread completed, so when a
// softmax warp sees S_h(k) the product PV_h(k - 2) is in O_h; PV_h(k - 1) may still be
// running, and the lazy O rescale (rare) waits for it first. Each row's visible keys within a
// block are three intervals (past, trunk, own branch), turned into a 32-bit mask per thread
// and unit.
// Warps: 0 TMA, 1 MMA, 2-9 softmax head 2p, 10-17 softmax head 2p+1 (576 threads), each softmax
// warp 16 rows with two threads per row (the 16x32bx2 TMEM access shape), so each SM
// sub-partition holds four softmax warps. The softmax warps are latency-bound rather than
// issue-bound (issue slots 40% busy with two softmax warps per sub-partition, 56% with four;
// configuration-2 batch: 128-key units with one thread per row 661, 64-key units 673, two
// threads per row 766 TFLOP/s). Measured and not kept: bf16 packing of P by integer rounding
// instead of the conversion instruction (-14%), scalar instead of packed f32x2 arithmetic
// (-4%), every exponential on the MUFU unit (-3%), S of a whole 128-key block per QK group
// (N = 128, which the tensor core reads its shared-memory operands for at full rate where
// N = 64 runs at two thirds) at the cost of the per-unit prefetch (-4.5%).
// TMEM: S_0 [0,64) [64,128), S_1 [128,192) [192,256) (P of a unit over the first 32
// columns of its buffer), O_0 [256, 256+D), O_1 [256+D, 256+2D).
template <int D>
struct PairCfg {
  static constexpr int NS = D <= 64 ? 3 : 2;
  static constexpr int CHUNKS = D / 64;
  static constexpr int Q_BYTES = CHUNKS * CHUNK;  // one head's 128 query rows
  static constexpr int KV_BYTES = CHUNKS * CHUNK;
  // Output staging: per softmax warp two 1 KB slots (16 rows x 32 bf16 columns each, one per
  // column half), written with the 64-byte swizzle and sent by TMA store.
  static constexpr int SLOT_BYTES = 16 * 64;
  static constexpr int SINK_BYTES = 16 * 2 * SLOT_BYTES;
  // 225.5 KB at D = 128: a second Q buffer (64 KB) does not fit.
  static constexpr int SMEM_USED = 2 * Q_BYTES + 2 * NS * KV_BYTES + SINK_BYTES + 1024 + 512;
  static constexpr int SMEM = SMEM_USED < 120 * 1024 ? 120 * 1024 : SMEM_USED;
  static constexpr int THREADS = 576;
};

// Shared-memory operand descriptors (128-byte swizzle) as two words: the low word holds the start
// address and the leading-dimension offset, the high word the 1024-byte stride offset, the
// sm100 version bit and the swizzle mode. The paired kernel's MMA issuer steps through an
// operand by adding to the low word only (shared addresses stay below 256 KB, so the 14-bit
// address field never carries), which keeps its instruction stream short: it shares an SM
// sub-partition with four busy softmax warps.
__device__ __forceinline__ uint32_t desc_lo(uint32_t saddr, uint32_t lbo) {
  return ((saddr & 0x3FFFFu) >> 4) | (((lbo >> 4) & 0x3FFFu) << 16);
}
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);

__device__ __forceinline__ void mma_ss_w(uint32_t d, uint32_t alo, uint32_t blo, uint32_t hi, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\tsetp.ne.b32 p, %4, 0;\n\tmov.b64 da, {%1, %5};\n\t"
      "mov.b64 db, {%2, %5};\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t}\n" ::"r"(d),
      "r"(alo), "r"(blo), "r"(idesc), "r"(acc), "r"(hi)
      : "memory");
}
__device__ __forceinline__ void mma_ts_w(uint32_t d, uint32_t a_tmem, uint32_t blo, uint32_t hi, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\tsetp.ne.b32 p, %4, 0;\n\tmov.b64 db, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %3, p;\n\t}\n" ::"r"(d),
      "r"(a_tmem), "r"(blo), "r"(idesc), "r"(acc), "r"(hi)
      : "memory");
}

template <int D>
__global__ void __launch_bounds__(576, 1)
    tree_attention_pair_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                               const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tpk,
                               const __grid_constant__ CUtensorMap tpv, const __grid_constant__ CUtensorMap to,
                               Params p, int n_items) {
  using C = PairCfg<D>;
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;  // [2 heads][Q_BYTES]
  uint8_t* sk = sq + 2 * C::Q_BYTES;
  uint8_t* sv = sk + NS * C::KV_BYTES;
  uint8_t* sink = sv + NS * C::KV_BYTES;  // 1024-byte aligned: Q and K/V stages are multiples of 8 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sink + C::SINK_BYTES);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;
  uint64_t* k_full = q_empty + 1;   // [NS]
  uint64_t* v_full = k_full + NS;
  uint64_t* k_empty = v_full + NS;
  uint64_t* v_empty = k_empty + NS;
  uint64_t* s_full = v_empty + NS;  // [head * 2 + buffer]
  uint64_t* p_full = s_full + 4;    // [head * 2 + buffer]
  uint64_t* pv_done = p_full + 4;   // [head * 2 + buffer]
  uint64_t* o_free = pv_done + 4;   // [head]: the epilogue finished reading O_h
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);

  const int npairs = p.n_heads / 2;
  const int rep = p.n_heads / p.n_kv_heads;
  const Tile* tiles = reinterpret_cast<const Tile*>(p.tiles);
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);
      mbar_init(&pv_done[b], 1);
    }
    for (int h = 0; h < 2; ++h) mbar_init(&o_free[h], 8);
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

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      uint32_t gb = 0, it = 0;
      bool ok = true;
      for (int kw = 0; ok; ++kw) {
        const int w = item_at(p, kw, n_items);
        if (w < 0) break;
        const Tile tile = tiles[w / npairs];
        const int head0 = 2 * (w % npairs), kvh = head0 / rep;
        const int nblk = tile.nblk_a + (tile.blk_b1 - tile.blk_b0);
        if (nblk == 0) continue;
        if (!mbar_wait(q_empty, (it & 1) ^ 1)) {
          report(p.status, kTimeoutEmpty);
          break;
        }
        mbar_expect_tx(q_full, 2 * C::Q_BYTES);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_3d(sq + h * C::Q_BYTES + c * CHUNK, &tq, q_full, c * 64, head0 + h, tile.row0);
        for (int j = 0; j < nblk; ++j, ++gb) {
          const int stage = gb % NS;
          const uint32_t ph = (gb / NS) & 1;
          const int b = j < tile.nblk_a ? j : tile.blk_b0 + (j - tile.nblk_a);
          const int kb = b * BN;
          const bool pool = kb < tile.ppad;
          const int row = pool ? p.pages[tile.page0 + b] * BN : tile.seg_start + (kb - tile.ppad);
          const CUtensorMap* mk = pool ? &tpk : &tk;
          const CUtensorMap* mv = pool ? &tpv : &tv;
          if (!mbar_wait(&k_empty[stage], ph ^ 1)) {
            report(p.status, kTimeoutEmpty);
            ok = false;
            break;
          }
          mbar_expect_tx(&k_full[stage], C::KV_BYTES);
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_3d(sk + stage * C::KV_BYTES + c * CHUNK, mk, &k_full[stage], c * 64, kvh, row);
          if (!mbar_wait(&v_empty[stage], ph ^ 1)) {
            report(p.status, kTimeoutEmpty);
            ok = false;
            break;
          }
          mbar_expect_tx(&v_full[stage], C::KV_BYTES);
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_3d(sv + stage * C::KV_BYTES + c * CHUNK, mv, &v_full[stage], c * 64, kvh, row);
        }
        ++it;
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_bf16(BM, 64, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(BM, D, false, true);
      const uint32_t hi = kDescHi;
      // S_h(k) = Q_h K[64 keys]^T into buffer k & 1 of head h; k counts the units of the item
      // whose first key block is this CTA's block g0.
      auto qk = [&](int h, uint32_t g0, int k, int nu) -> bool {
        const uint32_t g = g0 + (k >> 1);
        const int s = k & 1, st = g % NS;
        if (h == 0 && s == 0 && !mbar_wait(&k_full[st], (g / NS) & 1)) {
          report(p.status, kTimeoutFull);
          return false;
        }
        tc_fence_after();
        const uint32_t qlo = desc_lo(smem_u32(sq + h * C::Q_BYTES), 16);
        const uint32_t klo = desc_lo(smem_u32(sk + st * C::KV_BYTES) + s * 64 * 128, 16);  // key rows [64 s, +64)
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4;
          mma_ss_w(tmem + h * 128 + s * 64, qlo + off, klo + off, hi, idesc_qk, kk > 0);
        }
        mma_commit(&s_full[h * 2 + s]);
        if (h == 1) {
          if (s == 1) mma_commit(&k_empty[st]);
          if (k == nu - 1) mma_commit(q_empty);
        }
        return true;
      };
      // O_h += P_h(k) V[64 keys], P read from the first 32 columns of the unit's buffer.
      auto pv = [&](int h, uint32_t g0, int k, uint32_t it) -> bool {
        const uint32_t g = g0 + (k >> 1);
        const int s = k & 1, st = g % NS;
        if (k == 0 && !mbar_wait(&o_free[h], (it & 1) ^ 1)) {
          report(p.status, kTimeoutSoftmax);
          return false;
        }
        if (!mbar_wait(&p_full[h * 2 + s], g & 1)) {
          report(p.status, kTimeoutSoftmax);
          return false;
        }
        if (h == 0 && s == 0 && !mbar_wait(&v_full[st], (g / NS) & 1)) {
          report(p.status, kTimeoutFull);
          return false;
        }
        tc_fence_after();
        const uint32_t vlo = desc_lo(smem_u32(sv + st * C::KV_BYTES) + s * 64 * 128, CHUNK);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts_w(tmem + 256 + h * D, tmem + h * 128 + s * 64 + kk * 8, vlo + kk * (2048 >> 4), hi, idesc_pv,
                   (k > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&pv_done[h * 2 + s]);
        if (h == 1 && s == 1) mma_commit(&v_empty[st]);
        return true;
      };
      uint32_t gb = 0, it = 0;
      bool ok = true;
      for (int kw = 0; ok; ++kw) {
        const int w = item_at(p, kw, n_items);
        if (w < 0) break;
        const Tile tile = tiles[w / npairs];
        const int nu = 2 * (tile.nblk_a + (tile.blk_b1 - tile.blk_b0));
        if (nu == 0) continue;
        if (!mbar_wait(q_full, it & 1)) {
          report(p.status, kTimeoutFull);
          break;
        }
        // Head 2p's two units first: head 2p+1's softmax starts ~two QK products later, so the
        // heads' exponential phases (which share the MUFU unit) overlap less (three
        // configuration-2 batches: +0.3 to +2%, outputs bit-identical).
        ok = qk(0, gb, 0, nu) && qk(0, gb, 1, nu) && qk(1, gb, 0, nu) && qk(1, gb, 1, nu);
        for (int k = 0; ok && k < nu; ++k) {
          if (!(ok = pv(0, gb, k, it))) break;
          if (k + 2 < nu && !(ok = qk(0, gb, k + 2, nu))) break;
          if (!(ok = pv(1, gb, k, it))) break;
          if (k + 2 < nu && !(ok = qk(1, gb, k + 2, nu))) break;
        }
        gb += nu / 2;
        ++it;
      }
    }
  } else {
    // Warp w covers 16 rows of its TMEM lane quarter (w % 4) with two threads per row: thread
    // t < 16 takes row t and the first 32 keys of each unit (the first half of the O columns),
    // thread t + 16 the same row and the last 32 keys (the second half of O). The two halves of
    // a row share their maximum by one shuffle.
    const int sidx = warp - 2;        // 0..15
    const int hsel = sidx >> 3;       // 0: head 2p, 1: head 2p+1
    const int sub = warp & 3;         // TMEM lane quarter
    const int lh = (sidx >> 2) & 1;   // which 16 lanes of the quarter
    const int half = lane >> 4;       // key half of a unit, column half of O
    const int r0 = sub * 32 + lh * 16;  // first tile row of this warp
    const int r_in = r0 + (lane & 15);
    const uint32_t lane_base = static_cast<uint32_t>(r0) << 16;
    const uint32_t s_addr = tmem + lane_base + hsel * 128;
    const uint32_t o_addr = tmem + lane_base + 256 + hsel * D;
    const float sl2 = p.scale_log2;
    uint8_t* wslots = sink + sidx * 2 * C::SLOT_BYTES;  // per key half: 16 rows x 32 columns
    uint8_t* slot = wslots + half * C::SLOT_BYTES;
    uint32_t gb = 0;
    bool ok = true;
    for (int kw = 0; ok; ++kw) {
      const int w = item_at(p, kw, n_items);
      if (w < 0) break;
      const Tile tile = tiles[w / npairs];
      const int head = 2 * (w % npairs) + hsel;
      const int nblk = tile.nblk_a + (tile.blk_b1 - tile.blk_b0);
      if (nblk == 0) continue;
      const int row = tile.row0 + r_in;
      const bool valid = r_in < tile.nrows;
      const int qv = tile.q0v + r_in;
      const int own = valid ? tile.ppad + (p.row_own[row] - tile.seg_start) : tile.ppad;
      const int e_past = min(tile.past, qv + 1), e_trunk = min(tile.split, qv + 1);
      float m = -INFINITY, l = 0.f;  // m in log2 units (scaled); l over this thread's keys
      for (int j = 0; j < nblk && ok; ++j) {
        const uint32_t g = gb + j;
        const int b = j < tile.nblk_a ? j : tile.blk_b0 + (j - tile.nblk_a);
        const int kb = b * BN;
        const bool full = (kb + BN <= tile.past) ||
                          (kb >= tile.ppad && kb + BN <= tile.split && kb + BN - 1 <= tile.q0v);
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          // this thread's 32 keys of unit s: block columns [64 s + 32 half, + 32)
          const int base = kb + 64 * s + 32 * half;
          const uint32_t mw = full ? 0xffffffffu
                                   : (span_bits(-base, e_past - base) | span_bits(tile.ppad - base, e_trunk - base) |
                                      span_bits(own - base, qv + 1 - base));
          // warp-uniform path over both halves: 0 no key visible, 1 mixed, 2 every key visible
          const uint32_t cls = full ? 2u
                                    : (__all_sync(0xffffffffu, mw == 0xffffffffu)
                                           ? 2u
                                           : (__any_sync(0xffffffffu, mw != 0u) ? 1u : 0u));
          const uint32_t sb = s_addr + s * 64;
          if (!mbar_wait(&s_full[hsel * 2 + s], g & 1)) {
            report(p.status, kTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t x[32];
          tmem_ld16x2_x32<32>(sb, x);
          tmem_wait_ld_regs(x);
          float mx = -INFINITY;
          chunk_prep_u(x, mw, cls, mx);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float m_new = fmaxf(m, mx * sl2);
          bool rescale = false;
          float alpha = 1.f;
          if (m_new != -INFINITY) {
            if (m == -INFINITY) {
              m = m_new;
            } else if (m_new > m + 8.f) {
              alpha = fast_exp2(m - m_new);
              m = m_new;
              rescale = true;
            }
          }
          const float mu = m == -INFINITY ? 0.f : m;
          float sum = 0.f;
          {
            uint32_t pk[16];
            chunk_p_u(x, cls, sl2, mu, sum, pk);
            tmem_st16x2_x16<16>(sb, pk);  // P keys [0, 32) -> columns [0, 16), keys [32, 64) -> [16, 32)
          }
          l = l * alpha + sum;
          if (__any_sync(0xffffffffu, rescale)) {
            // O_h must hold the previous unit's product before it is scaled: PV_h of the
            // previous unit may still be running (the one before it has completed).
            const bool waited = s == 1 ? mbar_wait(&pv_done[hsel * 2], g & 1)
                                       : mbar_wait(&pv_done[hsel * 2 + 1], (g - 1) & 1);
            if (!waited) {
              report(p.status, kTimeoutMma);
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < D / 2; c += 32) {
              uint32_t o[32];
              tmem_ld16x2_x32<D / 2>(o_addr + c, o);
              tmem_wait_ld_regs(o);
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16x2_x32<D / 2>(o_addr + c, o);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[hsel * 2 + s]);
        }
      }
      if (!ok) break;
      const uint32_t last = gb + nblk - 1;
      if (!mbar_wait(&pv_done[hsel * 2 + 1], last & 1)) {
        report(p.status, kTimeoutMma);
        break;
      }
      tc_fence_after();
      const float lt = l + __shfl_xor_sync(0xffffffffu, l, 16);
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      // A warp whose 16 rows all belong to the tile sends each 16 x 32 piece through its
      // shared-memory slot by TMA store (whole lines, no per-row stores); the warp holding a
      // segment's ragged last rows stores its valid rows directly.
      const bool slab = r0 + 16 <= tile.nrows;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(row) * p.out_row + static_cast<int64_t>(head) * p.out_head;
#pragma unroll 1
      for (int c = 0; c < D / 2; c += 32) {
        uint32_t o[32];
        tmem_ld16x2_x32<D / 2>(o_addr + c, o);
        tmem_wait_ld_regs(o);
        uint32_t pkd[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pkd[i] = pack_bf16(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        const int col = half * (D / 2) + c;
        if (slab) {
          if (lane == 0) bulk_wait_read<0>();  // the previous stores from these slots have read them
          __syncwarp();
          // 64-byte swizzle: 16-byte unit u of row r sits at unit u ^ ((r >> 1) & 3)
          const int r = lane & 15;
          uint4* d4 = reinterpret_cast<uint4*>(slot + r * 64);
          const int sw = (r >> 1) & 3;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i ^ sw] = make_uint4(pkd[4 * i], pkd[4 * i + 1], pkd[4 * i + 2], pkd[4 * i + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&to, wslots, c, head, tile.row0 + r0);
            tma_store_3d(&to, wslots + C::SLOT_BYTES, D / 2 + c, head, tile.row0 + r0);
            bulk_commit();
          }
          __syncwarp();
        } else if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + col);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pkd[4 * i], pkd[4 * i + 1], pkd[4 * i + 2], pkd[4 * i + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[hsel]);
      gb += nblk;
    }
    if (lane == 0) bulk_wait_all();  // output stores done before the CTA's shared memory goes away
    tc_fence_before();
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch_pair(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tpk,
                const CUtensorMap& tpv, const CUtensorMap& to, const Params& p, int n_tiles, cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  DAN_CUDA(smem_limit_once(tree_attention_pair_kernel<D>, PairCfg<D>::SMEM, configured));
  const int items = n_tiles * (p.n_heads / 2);
  const int grid = p.sched ? p.sched_ctas : (items < sm_count() ? items : sm_count());
  tree_attention_pair_kernel<D><<<grid, PairCfg<D>::THREADS, PairCfg<D>::SMEM, stream>>>(tq, tk, tv, tpk, tpv, to,
                                                                                        p, items);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

static int rows_map(CUtensorMap* m, const void* base, int64_t row_stride, int64_t head_stride, int heads, int rows,
                    int d) {
  uint64_t dims[3] = {static_cast<uint64_t>(d), static_cast<uint64_t>(heads), static_cast<uint64_t>(rows)};
  uint64_t strides[2] = {static_cast<uint64_t>(head_stride) * 2, static_cast<uint64_t>(row_stride) * 2};
  uint32_t box[3] = {64, 1, 128};
  return make_tmap(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Output tiles: 32 columns x 1 head x ``box_rows`` rows per store (16 for both kernels), 64-byte
// swizzle.
static int out_map(CUtensorMap* m, const void* base, int64_t row_stride, int64_t head_stride, int heads, int rows,
                   int d, int box_rows) {
  uint64_t dims[3] = {static_cast<uint64_t>(d), static_cast<uint64_t>(heads), static_cast<uint64_t>(rows)};
  uint64_t strides[2] = {static_cast<uint64_t>(head_stride) * 2, static_cast<uint64_t>(row_stride) * 2};
  uint32_t box[3] = {32, 1, static_cast<uint32_t>(box_rows)};
  return make_tmap(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}

}  // namespace attn
}  // namespace dan

using namespace dan;

DAN_API int dan_tree_attention(const void* q, int64_t q_row, int64_t q_head, const void* k, int64_t k_row,
                               int64_t k_head, const void* v, int64_t v_row, int64_t v_head, const void* k_pool,
                               const void* v_pool, int64_t pool_row, int64_t pool_head, int pool_rows, void* out,
                               int64_t out_row, int64_t out_head, int n_rows, int n_heads, int n_kv_heads,
                               int head_dim, const int* tiles, int n_tiles, const int* row_own, const int* pages,
                               const int* schedule, int sched_ctas, float scale, int32_t* status, void* stream) {
  DAN_REQUIRE(n_rows > 0 && n_tiles >= 0, "tree_attention: n_rows=%d n_tiles=%d", n_rows, n_tiles);
  DAN_REQUIRE(!schedule || sched_ctas > 0, "tree_attention: a schedule needs its CTA count");
  DAN_REQUIRE(n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0,
              "tree_attention: %d query heads are not a multiple of %d kv heads", n_heads, n_kv_heads);
  DAN_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, "tree_attention: head_dim %d unsupported",
              head_dim);
  DAN_REQUIRE(n_tiles < 65536, "tree_attention: %d tiles exceed the grid limit", n_tiles);
  DAN_REQUIRE(out_head % 8 == 0 && out_row % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0,
              "tree_attention: output must be 16-byte aligned with strides that are multiples of 8");
  if (n_tiles == 0) return 0;
  CUtensorMap tq, tk, tv, tpk, tpv;
  int rc;
  if ((rc = attn::rows_map(&tq, q, q_row, q_head, n_heads, n_rows, head_dim))) return rc;
  if ((rc = attn::rows_map(&tk, k, k_row, k_head, n_kv_heads, n_rows, head_dim))) return rc;
  if ((rc = attn::rows_map(&tv, v, v_row, v_head, n_kv_heads, n_rows, head_dim))) return rc;
  if (k_pool && v_pool && pool_rows > 0) {
    if ((rc = attn::rows_map(&tpk, k_pool, pool_row, pool_head, n_kv_heads, pool_rows, head_dim))) return rc;
    if ((rc = attn::rows_map(&tpv, v_pool, pool_row, pool_head, n_kv_heads, pool_rows, head_dim))) return rc;
  } else {
    tpk = tk;
    tpv = tv;
  }
  attn::Params p{};
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_row = out_row;
  p.out_head = out_head;
  p.tiles = tiles;
  p.row_own = row_own;
  p.pages = pages;
  p.n_rows = n_rows;
  p.n_heads = n_heads;
  p.n_kv_heads = n_kv_heads;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  p.sched = schedule;
  p.sched_ctas = sched_ctas;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool paired = (n_heads / n_kv_heads) % 2 == 0 && head_dim <= 128;
  CUtensorMap to;
  if ((rc = attn::out_map(&to, out, out_row, out_head, n_heads, n_rows, head_dim, 16))) return rc;
  if (paired)
    return head_dim == 64 ? attn::launch_pair<64>(tq, tk, tv, tpk, tpv, to, p, n_tiles, s)
                          : attn::launch_pair<128>(tq, tk, tv, tpk, tpv, to, p, n_tiles, s);
  switch (head_dim) {
    case 64:
      return attn::launch<64>(tq, tk, tv, tpk, tpv, to, p, n_tiles, s);
    case 128:
      return attn::launch<128>(tq, tk, tv, tpk, tpv, to, p, n_tiles, s);
    default:
      return attn::launch<256>(tq, tk, tv, tpk, tpv, to, p, n_tiles, s);
  }
}
