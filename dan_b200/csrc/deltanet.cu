// Gated DeltaNet layers of the Qwen3.5 hybrid: causal depthwise conv + SiLU,
// the gated delta rule over the tree of runs, and the gated RMSNorm.
//
// Reference: dan/models/qwen3_5.py:161-298 (DeltaNet.forward, _phase,
// RecurrentLayout), delta_rule_torch 103-133, l2norm 99-100, and the fused
// gates / norms of dan/fused.py:51-56, 79-82.
//
// Tree runs: a segment's trunk runs from its initial state (zeros, or the
// prefix pool's state slot) after k-1 history rows (zeros, or the pool's conv
// tail); every branch runs from the trunk's final state, with the trunk's last
// k-1 rows as conv history. The chain kernel keeps one head's 128 x 128 state
// in TMEM (fp32) across the whole segment: it walks the trunk in chunks of 64
// tokens, writes the state at the prefix-save cut to the pool, keeps the
// trunk's final state as a second TMEM copy and forks each branch from it: the
// state never round-trips to HBM.
//
// Recurrence per token (delta_rule_torch, qwen3_5.py:103-133):
//   a = exp(g);  S <- a S;  u = beta (v - S^T k);  S <- S + k u^T;  o = S^T q
// with k, q l2-normalised (eps 1e-6) and q scaled by Dk^-0.5; evaluated per
// chunk in the WY form on the tensor cores (chunk_prep_kernel, then
// chunk_state_kernel, below).
#include "common.cuh"

#include <mutex>
#include <type_traits>

namespace dan {
namespace delta {

__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// Row code for the conv source: >= 0 packed row of ``src``; -1 a zero row; <= -2 row
// (-code - 2) of the history buffer ``hist``.
__device__ __forceinline__ const __nv_bfloat16* code_row(int code, const __nv_bfloat16* src, int64_t ld_src,
                                                         const __nv_bfloat16* hist, int64_t ld_hist) {
  if (code >= 0) return src + static_cast<int64_t>(code) * ld_src;
  if (code == -1) return nullptr;
  return hist + static_cast<int64_t>(-code - 2) * ld_hist;
}

// y[r, c] = silu(sum_j w[c, j] * ext_j) over ext = [prev3, prev2, prev1, row r] (qwen3_5.py:218-220).
// A block covers CONV_ROWS consecutive rows and 1024 channels (CONV_CPT = 4 per thread, one
// 8-byte vector per row, the 16 weights in registers) and loads all its rows, and the three
// packed rows before them, up front; a source that is a previous packed row (every trunk
// row's) comes from those registers, only branch starts and history rows are gathered. Four
// channels per thread (rather than eight) and 12 rows keep a thread at 64 registers, so four
// blocks share an SM and one block's loads overlap another's SiLU (exp and reciprocal on the
// conversion unit). Graph-timed on a 7189-row configuration-4 batch (8192 channels): 58.8 us,
// against 72.0 with eight channels, 16 rows and two blocks per SM (the halo rows loaded in
// the row loop), 69.8 with the halo up front, 62.6 with eight channels and 8 rows at three
// blocks per SM (spilling).
constexpr int CONV_ROWS = 12, CONV_CPT = 4;
// (row, head) items per warp of the gated norm at dv = 128; graph-timed on 7189 x 32 x 128:
// 1 / 2 / 4 / 8 items = 49.2 / 44.6 / 49.1 / 58.8 us (one item per warp before: 48.0).
constexpr int GNORM_ITEMS = 2;
__global__ void __launch_bounds__(256, 4) causal_conv_kernel(const __nv_bfloat16* src, int64_t ld_src,
                                                          const __nv_bfloat16* hist, int64_t ld_hist,
                                                          const __nv_bfloat16* w, const int* prev,
                                                          __nv_bfloat16* out, int64_t ld_out, int rows, int channels) {
  // tail threads redo the last CONV_CPT channels
  const int c0 = min((blockIdx.y * blockDim.x + threadIdx.x) * CONV_CPT, channels - CONV_CPT);
  float wf[CONV_CPT][4];  // weights [C, 4]: CONV_CPT channels x 4 taps
  {
    uint4 wv[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) wv[i] = __ldg(reinterpret_cast<const uint4*>(w + static_cast<int64_t>(c0) * 4) + i);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(wv);
#pragma unroll
    for (int t = 0; t < CONV_CPT; ++t)
#pragma unroll
      for (int j = 0; j < 4; ++j) wf[t][j] = __bfloat162float(we[t * 4 + j]);
  }
  const int r0 = blockIdx.x * CONV_ROWS;
  const int nr = min(CONV_ROWS, rows - r0);
  __shared__ int codes[CONV_ROWS * 3];
  if (threadIdx.x < nr * 3) codes[threadIdx.x] = prev[3 * r0 + threadIdx.x];
  uint2 cur[CONV_ROWS], halo[3];  // every load issued before any is used; halo[k] = row r0 - 3 + k
#pragma unroll
  for (int i = 0; i < CONV_ROWS; ++i)
    cur[i] = __ldg(reinterpret_cast<const uint2*>(src + static_cast<int64_t>(r0 + min(i, nr - 1)) * ld_src + c0));
#pragma unroll
  for (int k = 0; k < 3; ++k)
    halo[k] = __ldg(reinterpret_cast<const uint2*>(src + static_cast<int64_t>(max(r0 - 3 + k, 0)) * ld_src + c0));
  __syncthreads();
#pragma unroll
  for (int i = 0; i < CONV_ROWS; ++i) {
    if (i >= nr) break;
    const int r = r0 + i;
    const int* pr = codes + 3 * i;
    uint2 e[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int code = pr[j];
      if (i > j && code == r - 1 - j) {  // a previous packed row of this block: in registers
        e[j] = cur[i - 1 - j];
      } else if (i <= j && r - 1 - j >= 0 && code == r - 1 - j) {  // one of the three rows before it
        e[j] = halo[i + 2 - j];
      } else {
        const __nv_bfloat16* row = code_row(code, src, ld_src, hist, ld_hist);
        e[j] = row ? __ldg(reinterpret_cast<const uint2*>(row + c0)) : make_uint2(0, 0);
      }
    }
    const __nv_bfloat16* x0 = reinterpret_cast<const __nv_bfloat16*>(&e[2]);  // tap 0: third previous row
    const __nv_bfloat16* x1 = reinterpret_cast<const __nv_bfloat16*>(&e[1]);
    const __nv_bfloat16* x2 = reinterpret_cast<const __nv_bfloat16*>(&e[0]);
    const __nv_bfloat16* x3 = reinterpret_cast<const __nv_bfloat16*>(&cur[i]);
    uint2 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int t = 0; t < CONV_CPT / 2; ++t) {
      float y[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int ch = 2 * t + u;
        float acc = wf[ch][0] * __bfloat162float(x0[ch]);
        acc += wf[ch][1] * __bfloat162float(x1[ch]);
        acc += wf[ch][2] * __bfloat162float(x2[ch]);
        acc += wf[ch][3] * __bfloat162float(x3[ch]);
        y[u] = silu(acc);
      }
      op[t] = pack_bf16(y[0], y[1]);
    }
    *reinterpret_cast<uint2*>(out + static_cast<int64_t>(r) * ld_out + c0) = o;
  }
}

// dst[i] = row(codes[i]) (zero rows for -1): conv tails of prefix saves.
__global__ void gather_rows_kernel(const __nv_bfloat16* src, int64_t ld_src, const __nv_bfloat16* hist,
                                   int64_t ld_hist, const int* codes, __nv_bfloat16* dst, int64_t ld_dst, int cols) {
  const int i = blockIdx.x;
  const __nv_bfloat16* s = code_row(codes[i], src, ld_src, hist, ld_hist);
  __nv_bfloat16* d = dst + static_cast<int64_t>(i) * ld_dst;
  for (int c = threadIdx.x * 8; c < cols; c += blockDim.x * 8)
    *reinterpret_cast<uint4*>(d + c) = s ? *reinterpret_cast<const uint4*>(s + c) : make_uint4(0, 0, 0, 0);
}

// Segment record (int32 x 8): trunk_start, trunk_len, cut, init_slot, save_slot, branch0, n_branches,
// first chunk. Branch record (int32 x 4): start, len, first chunk, 0.
struct Seg {
  int trunk_start, trunk_len, cut, init_slot, save_slot, branch0, n_branches, pad;
};

struct ScanParams {
  const __nv_bfloat16* q;  // conv output, q of k-head kh at q + row * ld_qkv + kh * dk
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ld_qkv;
  const __nv_bfloat16* b;  // in_proj b / a columns, [rows, hv] with row stride ld_ba
  const __nv_bfloat16* a;
  int64_t ld_ba;
  const float* a_log;    // [hv]; nullptr: the gates are given (b holds beta, g_given the log decay)
  const float* dt_bias;  // [hv]
  const float* g_given;  // [rows, hv] fp32 log decay, row stride ld_g (when a_log is nullptr)
  int64_t ld_g;
  const Seg* segs;
  const int* branches;
  float* state_pool;  // [slots, hv, dk, dv] of this layer (slot stride given)
  int64_t slot_stride;
  __nv_bfloat16* out;  // [rows, hv, dv]
  int64_t ld_out;
  int hk, hv;
  float q_scale;
  const int* chunks;  // [n_chunks, 2]: first row, rows
  int n_chunks;
  uint8_t* scratch;   // chunk records (REC_V per chunk and value head, REC_K per chunk and key head)
  int32_t* status;
  // Launch subsets (zero for a launch over everything): the pre-pass's chunk of block x is
  // chunk_base + x, then moved past [skip_at, skip_at + skip_len); the chain's segment of
  // block y is seg_base + y.
  int chunk_base, skip_at, skip_len, seg_base;
};

constexpr int DK = 128;

// ---------------------------------------------------------------------------------
// Chunked gated delta rule on the tensor cores (bf16 operands, fp32 accumulation: mma.sync
// m16n8k16 in the pre-pass, tcgen05 in the chain). Runs are cut into chunks of CH = 64 tokens. With Γ_t the cumulative log
// decay inside a chunk (γ_t = e^Γ_t), the token recurrence S_t = d_t S_{t-1} + k_t u_t^T,
// u_t = β_t (v_t - k_t^T d_t S_{t-1}), o_t = q_t^T S_t unrolls over a chunk that starts from
// state S0 to (the WY form; every decay factor is e^{difference} <= 1)
//   A  = strictly_lower(β_t e^{Γ_t-Γ_s} k_t.k_s),  T = (I + A)^-1,  T' = T diag(β)
//   U  = T'V - W S0,  W = T' diag(γ) K
//   O  = diag(γ) Q S0 + P U,  P = (e^{Γ_t-Γ_s} q_t.k_s for s <= t)
//   S  = γ_C S0 + K^T diag(e^{Γ_C-Γ_t}) U
// chunk_prep_kernel computes everything that does not depend on S0 for all chunks at once
// (one CTA per chunk and value head): normalised q and k, gates, P, T (fp32, 16 x 16
// diagonal blocks by substitution then two merge levels), -W, diag(γ) q̂ and T'V, into a
// scratch buffer. chunk_state_kernel then walks each segment's chunks in order (one CTA per
// value head and segment) doing only U, O and the state update, with the fp32 state in TMEM
// for the whole segment (see the chain's own comment below).
constexpr int CH = 64;
constexpr int LDW = DK + 8;  // bf16 row stride of 128-wide tiles: 272 B, ldmatrix rows on distinct banks
constexpr int LDN = CH + 8;  // bf16 row stride of 64-wide tiles
constexpr int LDF = CH + 1;  // fp32 row stride of 64 x 64 tiles
constexpr int LDT = CH + 4;  // fp32 row stride of T: 16-byte rows for the merges' vector loads
constexpr int LDY = 36;      // fp32 row stride of the merges' 32-wide scratch

// Scratch records, laid out exactly as the chain kernel's shared memory so a chunk loads with
// a few bulk copies: per (chunk, value head) -W and diag(γ) q̂ [64 rows t][128] and P [64][64]
// in the 128-byte swizzled row layout of tcgen05 operands (64-column chunks of 8 KB), T'V
// [64][LDW] bf16, and γ_t, e^{Γ_C-Γ_t}, e^{Γ_C} (fp32 x 64 each); per (chunk, key head) k̂
// [64 rows][128], swizzled the same way.
constexpr int64_t REC_W = 0, REC_QG = 16384, REC_P = 32768, REC_TV = 40960;
constexpr int64_t REC_SC = REC_TV + CH * LDW * 2;  // 58368
constexpr int64_t REC_V = REC_SC + 3 * CH * 4;     // 59136 B
constexpr int64_t REC_K = 16384;

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Fragment addresses (lane l) of a 16 x 16 A tile at (r0, k0) of a row-major [rows][ld] array;
// of A = X^T at (m0, k0) from X stored [k][ld]; of two 16 x 8 B tiles (n0, n0 + 8) at k0 from
// B^T stored [n][ld] (rows n); and from B stored [k][ld] (rows k).
__device__ __forceinline__ const __nv_bfloat16* a_rows(const __nv_bfloat16* x, int ld, int r0, int k0, int l) {
  return x + (r0 + (l & 15)) * ld + k0 + ((l >> 4) << 3);
}
__device__ __forceinline__ const __nv_bfloat16* a_cols(const __nv_bfloat16* x, int ld, int m0, int k0, int l) {
  return x + (k0 + (l & 7) + ((l >> 4) << 3)) * ld + m0 + (((l >> 3) & 1) << 3);
}
__device__ __forceinline__ const __nv_bfloat16* b_nrows(const __nv_bfloat16* x, int ld, int n0, int k0, int l) {
  return x + (n0 + (l & 7) + ((l >> 4) << 3)) * ld + k0 + (((l >> 3) & 1) << 3);
}
__device__ __forceinline__ const __nv_bfloat16* b_krows(const __nv_bfloat16* x, int ld, int k0, int n0, int l) {
  return x + (k0 + (l & 15)) * ld + n0 + ((l >> 4) << 3);
}
__device__ __forceinline__ void st_bf2(__nv_bfloat16* p, float x, float y) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16(x, y);
}

struct PrepSmem {
  __nv_bfloat16 qn[CH * LDW];  // q̂, later -W
  __nv_bfloat16 kn[CH * LDW];  // k̂
  __nv_bfloat16 v[CH * LDW];   // v, later T'V
  float a[CH * LDF];           // A
  float tf[CH * LDT];          // T
  __nv_bfloat16 tb[CH * LDN];  // T diag(β) (fp32 merge scratch before that)
  __nv_bfloat16 tg[CH * LDN];  // T diag(βγ)
  __nv_bfloat16 pb[CH * LDN];  // P
  float gam[CH], eg[CH], beta[CH], graw[CH];
};

// A padded [64 rows][ld] bf16 tile of shared memory (``chunks`` x 64 columns) to global memory
// in the 128-byte swizzled row layout (per 64-column chunk, row r's 16-byte unit u at
// r * 128 + ((u ^ (r & 7)) * 16)).
__device__ __forceinline__ void copy_out_sw128(uint8_t* dst, const __nv_bfloat16* src, int ld, int chunks) {
  for (int e = threadIdx.x; e < CH * 8 * chunks; e += blockDim.x) {
    const int r = e / (8 * chunks), j = e % (8 * chunks), ch = j >> 3, u = j & 7;
    *reinterpret_cast<uint4*>(dst + ch * 8192 + r * 128 + ((u ^ (r & 7)) << 4)) =
        *reinterpret_cast<const uint4*>(src + r * ld + 8 * j);
  }
}

__global__ void __launch_bounds__(256, 2) chunk_prep_kernel(ScanParams p) {
  extern __shared__ __align__(16) uint8_t dsm[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(dsm);
  const int h = blockIdx.y;
  int ci = p.chunk_base + static_cast<int>(blockIdx.x);
  if (ci >= p.skip_at) ci += p.skip_len;
  const int row0 = p.chunks[2 * ci], nt = p.chunks[2 * ci + 1];
  const int per = p.hv / p.hk, kh = h / per;
  const bool owner = h % per == 0;  // writes this key head's q̂ and k̂
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const bool given = p.a_log == nullptr;
  const float a_neg = given ? 0.f : -__expf(p.a_log[h]), dtb = given ? 0.f : p.dt_bias[h];
  uint8_t* rv = p.scratch + (static_cast<int64_t>(ci) * p.hv + h) * REC_V;
  uint8_t* rk = p.scratch + static_cast<int64_t>(p.n_chunks) * p.hv * REC_V + (static_cast<int64_t>(ci) * p.hk + kh) * REC_K;
  // ---- stage: raw q, k, v rows by cp.async (16 B per thread step, all in flight), gates; T cleared
  {
    const __nv_bfloat16* srcs[3] = {p.q + kh * DK, p.k + kh * DK, p.v + h * DK};
    __nv_bfloat16* dsts[3] = {sm.qn, sm.kn, sm.v};
    const int c8 = (tid & 15) * 8;
#pragma unroll
    for (int w = 0; w < 3; ++w) {
      const __nv_bfloat16* src = srcs[w] + static_cast<int64_t>(row0) * p.ld_qkv + c8;
#pragma unroll
      for (int t = tid >> 4; t < CH; t += 16) {  // 16 threads per row, 16 rows per pass
        if (t < nt)
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dsts[w] + t * LDW + c8)),
                       "l"(src + static_cast<int64_t>(t) * p.ld_qkv)
                       : "memory");
      }
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if (lane < 8) {
    const int t = warp * 8 + lane;
    float bb = 0.f, gg = 0.f;
    if (t < nt) {
      const int64_t row = row0 + t;
      if (given) {
        bb = __bfloat162float(p.b[row * p.ld_ba + h]);
        gg = p.g_given[row * p.ld_g + h];
      } else {
        bb = 1.f / (1.f + __expf(-__bfloat162float(p.b[row * p.ld_ba + h])));
        gg = a_neg * softplus(__bfloat162float(p.a[row * p.ld_ba + h]) + dtb);
      }
    }
    sm.beta[t] = bb;
    sm.graw[t] = gg;
  }
  for (int e = tid; e < (CH - nt) * (DK / 8); e += blockDim.x) {  // rows past the chunk: zero
    const int t = nt + e / (DK / 8), c8 = (e % (DK / 8)) * 8;
    *reinterpret_cast<uint4*>(&sm.qn[t * LDW + c8]) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(&sm.kn[t * LDW + c8]) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(&sm.v[t * LDW + c8]) = make_uint4(0, 0, 0, 0);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // l2 norms in place (q also scaled), a warp's 8 rows interleaved
    const int t = warp * 8 + i;      // (rows past the chunk are zero and stay zero)
    uint2* qp = reinterpret_cast<uint2*>(&sm.qn[t * LDW + lane * 4]);
    uint2* kp = reinterpret_cast<uint2*>(&sm.kn[t * LDW + lane * 4]);
    const uint2 qw = *qp, kw = *kp;
    const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qw);
    const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kw);
    const float2 qa = __bfloat1622float2(q2[0]), qb = __bfloat1622float2(q2[1]);
    const float2 ka = __bfloat1622float2(k2[0]), kb = __bfloat1622float2(k2[1]);
    float sq = qa.x * qa.x + qa.y * qa.y + qb.x * qb.x + qb.y * qb.y;
    float sk = ka.x * ka.x + ka.y * ka.y + kb.x * kb.x + kb.y * kb.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    const float nq = rsqrtf(sq + 1e-6f) * p.q_scale, nk = rsqrtf(sk + 1e-6f);
    *qp = make_uint2(pack_bf16(qa.x * nq, qa.y * nq), pack_bf16(qb.x * nq, qb.y * nq));
    *kp = make_uint2(pack_bf16(ka.x * nk, ka.y * nk), pack_bf16(kb.x * nk, kb.y * nk));
  }
  for (int i = tid; i < CH * LDT; i += blockDim.x) sm.tf[i] = 0.f;
  __syncthreads();
  if (owner) copy_out_sw128(rk, sm.kn, LDW, 2);
  if (warp == 0) {  // Γ: inclusive prefix sum of the log decays
    const float v0 = sm.graw[2 * lane], v1 = sm.graw[2 * lane + 1];
    float incl = v0 + v1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    sm.gam[2 * lane] = incl - v1;
    sm.gam[2 * lane + 1] = incl;
    sm.eg[2 * lane] = __expf(incl - v1);
    sm.eg[2 * lane + 1] = __expf(incl);
  }
  __syncthreads();
  const float gc = sm.gam[nt - 1];
  {  // scalars: γ_t, e^{Γ_C-Γ_t}, e^{Γ_C}
    float* sc = reinterpret_cast<float*>(rv + REC_SC);
    if (tid < CH) {
      sc[tid] = sm.eg[tid];
      sc[CH + tid] = __expf(gc - sm.gam[tid]);
      sc[2 * CH + tid] = __expf(gc);
    }
  }
  for (int e = tid; e < CH * 16; e += blockDim.x) {  // diag(γ) q̂, swizzled rows
    const int r = e >> 4, j = e & 15, ch = j >> 3, u = j & 7;
    const uint4 qv = *reinterpret_cast<const uint4*>(&sm.qn[r * LDW + 8 * j]);
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
    const float gr = sm.eg[r];
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw[i]));
      o[i] = pack_bf16(f.x * gr, f.y * gr);
    }
    *reinterpret_cast<uint4*>(rv + REC_QG + ch * 8192 + r * 128 + ((u ^ (r & 7)) << 4)) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
  // ---- K K^T -> A and Q K^T -> P (warp: rows [16 tm, +16), columns [32 sh, +32))
  {
    // 16-column blocks 2 sh + np past the warp's row block tm lie above the diagonal, where A
    // and P are masked to zero: their products are skipped (warp-uniform).
    const int tm = warp & 3, sh = warp >> 2;
    const int nb = tm - 2 * sh + 1;  // column blocks of this warp at or below the diagonal (<= 2)
    float G[4][4] = {}, Pq[4][4] = {};
#pragma unroll 1
    for (int kk = 0; nb > 0 && kk < DK / 16; ++kk) {
      uint32_t ak[4], aq[4];
      ldsm4(ak, a_rows(sm.kn, LDW, 16 * tm, 16 * kk, lane));
      ldsm4(aq, a_rows(sm.qn, LDW, 16 * tm, 16 * kk, lane));
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        if (np >= nb) break;
        uint32_t b[4];
        ldsm4(b, b_nrows(sm.kn, LDW, 32 * sh + 16 * np, 16 * kk, lane));
        mma16816(G[2 * np], ak, b[0], b[1]);
        mma16816(G[2 * np + 1], ak, b[2], b[3]);
        mma16816(Pq[2 * np], aq, b[0], b[1]);
        mma16816(Pq[2 * np + 1], aq, b[2], b[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = 16 * tm + g + 8 * hh, s = 32 * sh + 8 * j + 2 * c;
        const float gt = sm.gam[t], bt = sm.beta[t];
        float av[2], pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float dec = (s + e <= t) ? __expf(gt - sm.gam[s + e]) : 0.f;
          av[e] = (s + e < t) ? bt * dec * G[j][2 * hh + e] : 0.f;
          pv[e] = dec * Pq[j][2 * hh + e];
        }
        sm.a[t * LDF + s] = av[0];
        sm.a[t * LDF + s + 1] = av[1];
        st_bf2(&sm.pb[t * LDN + s], pv[0], pv[1]);
      }
    }
  }
  __syncthreads();
  copy_out_sw128(rv + REC_P, sm.pb, LDN, 1);
  // ---- T = (I + A)^-1: diagonal 16 x 16 blocks by forward substitution (thread: one column)
  if (tid < 64) {
    const int d = tid >> 4, j = tid & 15;
    float x[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float acc = (t == j) ? 1.f : 0.f;
#pragma unroll
      for (int s2 = 0; s2 < t; ++s2) acc -= sm.a[(16 * d + t) * LDF + 16 * d + s2] * x[s2];
      x[t] = acc;
      sm.tf[(16 * d + t) * LDT + 16 * d + j] = acc;
    }
  }
  __syncthreads();
  float* ysc = reinterpret_cast<float*>(sm.tb);  // 32 x LDY fp32 scratch
  // The merges read rows of T and of the scratch as 8- / 16-byte vectors (LDT, LDY: 16-byte
  // rows); each output still accumulates over k in order.
  {  // level 1: T[d+1][d] = -T[d+1][d+1] A[d+1][d] T[d][d] for d = 0, 2
    const int q = tid >> 7, r = (tid >> 3) & 15, cc = (tid & 7) * 2, d = 2 * q;
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float av = sm.a[(16 * (d + 1) + r) * LDF + 16 * d + k];
      const float2 t2 = *reinterpret_cast<const float2*>(&sm.tf[(16 * d + k) * LDT + 16 * d + cc]);
      y0 += av * t2.x;
      y1 += av * t2.y;
    }
    *reinterpret_cast<float2*>(&ysc[(q * 16 + r) * LDY + cc]) = make_float2(y0, y1);
    __syncthreads();
    float x0 = 0.f, x1 = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float tv = sm.tf[(16 * (d + 1) + r) * LDT + 16 * (d + 1) + k];
      const float2 y2 = *reinterpret_cast<const float2*>(&ysc[(q * 16 + k) * LDY + cc]);
      x0 -= tv * y2.x;
      x1 -= tv * y2.y;
    }
    *reinterpret_cast<float2*>(&sm.tf[(16 * (d + 1) + r) * LDT + 16 * d + cc]) = make_float2(x0, x1);
  }
  __syncthreads();
  {  // level 2: T[32:64][0:32] = -T[32:64][32:64] A[32:64][0:32] T[0:32][0:32]
    const int r = tid >> 3, cq = (tid & 7) * 4;
    float y[4] = {};
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float av = sm.a[(32 + r) * LDF + k];
      const float4 t4 = *reinterpret_cast<const float4*>(&sm.tf[k * LDT + cq]);
      y[0] += av * t4.x;
      y[1] += av * t4.y;
      y[2] += av * t4.z;
      y[3] += av * t4.w;
    }
    *reinterpret_cast<float4*>(&ysc[r * LDY + cq]) = make_float4(y[0], y[1], y[2], y[3]);
    __syncthreads();
    float x[4] = {};
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float tv = sm.tf[(32 + r) * LDT + 32 + k];
      const float4 y4 = *reinterpret_cast<const float4*>(&ysc[k * LDY + cq]);
      x[0] -= tv * y4.x;
      x[1] -= tv * y4.y;
      x[2] -= tv * y4.z;
      x[3] -= tv * y4.w;
    }
    *reinterpret_cast<float4*>(&sm.tf[(32 + r) * LDT + cq]) = make_float4(x[0], x[1], x[2], x[3]);
  }
  __syncthreads();
  for (int e = tid; e < CH * CH / 2; e += blockDim.x) {  // T' = T diag(β) and T diag(βγ), bf16
    const int t = e >> 5, s2 = (e & 31) * 2;
    const float2 tt = *reinterpret_cast<const float2*>(&sm.tf[t * LDT + s2]);
    const float t0 = tt.x * sm.beta[s2], t1 = tt.y * sm.beta[s2 + 1];
    st_bf2(&sm.tb[t * LDN + s2], t0, t1);
    st_bf2(&sm.tg[t * LDN + s2], t0 * sm.eg[s2], t1 * sm.eg[s2 + 1]);
  }
  __syncthreads();
  // ---- T'V and W = T diag(βγ) K (warp: rows [16 tm, +16), columns [64 tn, +64)); T is lower
  // triangular, so row block tm only meets the key blocks kk <= tm.
  const int tm = warp & 3, tn = warp >> 2;
  float au[8][4] = {}, aw[8][4] = {};
#pragma unroll 1
  for (int kk = 0; kk <= tm; ++kk) {
    uint32_t a1[4], a2[4];
    ldsm4(a1, a_rows(sm.tb, LDN, 16 * tm, 16 * kk, lane));
    ldsm4(a2, a_rows(sm.tg, LDN, 16 * tm, 16 * kk, lane));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm4t(b, b_krows(sm.v, LDW, 16 * kk, 64 * tn + 16 * np, lane));
      mma16816(au[2 * np], a1, b[0], b[1]);
      mma16816(au[2 * np + 1], a1, b[2], b[3]);
      ldsm4t(b, b_krows(sm.kn, LDW, 16 * kk, 64 * tn + 16 * np, lane));
      mma16816(aw[2 * np], a2, b[0], b[1]);
      mma16816(aw[2 * np + 1], a2, b[2], b[3]);
    }
  }
  __syncthreads();  // v and q̂ buffers are free: T'V -> v, -W -> qn
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int t = 16 * tm + g, col = 64 * tn + 8 * j + 2 * c;
    st_bf2(&sm.v[t * LDW + col], au[j][0], au[j][1]);
    st_bf2(&sm.v[(t + 8) * LDW + col], au[j][2], au[j][3]);
    st_bf2(&sm.qn[t * LDW + col], -aw[j][0], -aw[j][1]);
    st_bf2(&sm.qn[(t + 8) * LDW + col], -aw[j][2], -aw[j][3]);
  }
  __syncthreads();
  copy_out_sw128(rv + REC_W, sm.qn, LDW, 2);
  for (int e = tid; e < CH * LDW / 8; e += blockDim.x)  // T'V [64][LDW]
    reinterpret_cast<uint4*>(rv + REC_TV)[e] = reinterpret_cast<const uint4*>(sm.v)[e];
}

// ---------------------------------------------------------------------------------
// The chain on the tensor cores (tcgen05, accumulators in TMEM): one CTA per (value head,
// segment) walks the segment's chunks in order. The state is held transposed, S^T [value
// column c = TMEM lane][key k] in fp32, so every product of a chunk is an M = 128 MMA over
// the head's 128 value columns with the A operand in TMEM:
//   U^T  = S0^T (-W)^T             A = S0^T (bf16), B = -W           (rows t, K = k)
//   U    = T'V + U^T^T             warps: bf16 U^T and Us^T = U^T diag(e^{Γ_C-Γ_t})
//   S^T  = γ_C S0^T + Us^T K       warps scale S^T first; B = K as an MN-major operand
//   O^T  = S0^T (diag(γ) Q)^T + U^T P^T
// TMEM columns: S^T [0,128), the trunk's final state F [128,256), U^T fp32 [256,320), O^T
// [320,384), S0^T bf16 [384,448), U^T bf16 [448,480), Us^T bf16 [480,512).
// Warps 0-3 (thread = value column = TMEM lane) convert between the products and stage O; warp
// 4 issues the bulk copies (three chunks in flight), the MMAs and O's TMA stores. Per chunk:
//   warps: S^T -> S0^T bf16 and S^T *= γ_C (after the previous chunk's S product); read the
//          previous chunk's O^T
//   MMA:   U^T
//   warps: U^T + T'V -> U^T, Us^T bf16; stage the previous O, transposed, in its chunk buffer
//   MMA:   S^T += Us^T K, then O^T; TMA store of the previous O, then the next bulk copies
// The products take ~900 tensor-core cycles per chunk; the TMEM round trips of the two
// conversions (load, wait, convert, store, wait) set the period (~3.7k cycles on a
// configuration-4 batch; eight conversion warps with half the work each measured no faster).
// The chain this replaces (mma.sync, which runs at a quarter of tcgen05's rate on B200: 2048 vs
// 8192 bf16 FLOP per clock and SM, with 128 x 64 of the state per CTA in registers) took 161 us
// on that batch, this one 152 us.
struct ChainBuf {               // one chunk's inputs; MMA operands 1024-byte aligned
  __nv_bfloat16 w[CH * DK];     // -W, rows t, 128-byte swizzle (two 64-column chunks)
  __nv_bfloat16 qg[CH * DK];    // diag(γ) q̂, same layout
  __nv_bfloat16 kn[CH * DK];    // k̂, same layout
  __nv_bfloat16 p[CH * CH];     // P, rows t, 128-byte swizzle
  __nv_bfloat16 tv[CH * LDW];   // T'V, row-major with padded rows
  float eg[CH], ws[CH], ec[CH];
  uint8_t pad[256];
};
static_assert(sizeof(ChainBuf) % 1024 == 0, "chunk buffers keep 1024-byte alignment");
struct ChainSmem {
  ChainBuf buf[3];
  uint64_t full[3];  // per buffer: the chunk's bulk copies landed
  uint64_t mma_u, mma_s, mma_o, conv_s, conv_u;
  uint64_t staged;   // the previous chunk's O left its buffer (staged there for coalesced stores)
  uint32_t tmem_slot;
};
constexpr uint32_t CHAIN_TX = 3 * 16384 + 8192 + CH * LDW * 2 + 3 * CH * 4;
constexpr int CHAIN_SMEM = static_cast<int>(sizeof(ChainSmem)) + 1024;  // + alignment of the base
static_assert(CHAIN_SMEM <= 232448, "the chain kernel's shared memory exceeds 227 KB");

enum StateSrc { kSrcZero = 0, kSrcPool = 1, kSrcTmemS = 2, kSrcTmemF = 3 };

__global__ void __launch_bounds__(160, 1) chunk_state_kernel(const __grid_constant__ CUtensorMap tout, ScanParams p) {
  extern __shared__ uint8_t dsm_raw[];
  ChainSmem& sm = *reinterpret_cast<ChainSmem*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const int h = blockIdx.x, kh = h / (p.hv / p.hk);
  const Seg sg = p.segs[p.seg_base + static_cast<int>(blockIdx.y)];
  const int warp = warp_id(), lane = lane_id();
  int total = (sg.cut + CH - 1) / CH + (sg.trunk_len - sg.cut + CH - 1) / CH;
  for (int bi = 0; bi < sg.n_branches; ++bi) total += (p.branches[4 * (sg.branch0 + bi) + 1] + CH - 1) / CH;
  const int c0 = sg.pad;  // first chunk of the segment
  const int n_runs = 2 + sg.n_branches;
  auto run_len = [&](int ri) {
    return ri == 0 ? sg.cut : (ri == 1 ? sg.trunk_len - sg.cut : p.branches[4 * (sg.branch0 + ri - 2) + 1]);
  };
  if (threadIdx.x == 0) {
    for (int b = 0; b < 3; ++b) mbar_init(&sm.full[b], 1);
    mbar_init(&sm.mma_u, 1);
    mbar_init(&sm.mma_s, 1);
    mbar_init(&sm.mma_o, 1);
    mbar_init(&sm.conv_s, 4);
    mbar_init(&sm.conv_u, 4);
    mbar_init(&sm.staged, 4);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_slot;

  if (warp == 4) {
    if (elect_one()) {
      auto load = [&](int i) {
        ChainBuf& b = sm.buf[i % 3];
        const int ci = c0 + i;
        const uint8_t* rv = p.scratch + (static_cast<int64_t>(ci) * p.hv + h) * REC_V;
        const uint8_t* rk = p.scratch + static_cast<int64_t>(p.n_chunks) * p.hv * REC_V +
                            (static_cast<int64_t>(ci) * p.hk + kh) * REC_K;
        fence_proxy_async();  // this buffer's previous generic reads before the async writes
        mbar_expect_tx(&sm.full[i % 3], CHAIN_TX);
        bulk_load(b.w, rv + REC_W, 16384, &sm.full[i % 3]);
        bulk_load(b.qg, rv + REC_QG, 16384, &sm.full[i % 3]);
        bulk_load(b.kn, rk, 16384, &sm.full[i % 3]);
        bulk_load(b.p, rv + REC_P, 8192, &sm.full[i % 3]);
        bulk_load(b.tv, rv + REC_TV, CH * LDW * 2, &sm.full[i % 3]);
        bulk_load(b.eg, rv + REC_SC, 3 * CH * 4, &sm.full[i % 3]);
      };
      // chunk j's O, once the converting warps staged it in the chunk's -W slot: whole chunks by
      // TMA store (the staging read before the buffer is reloaded), partial ones were stored by
      // the warps themselves
      auto store_staged = [&](int j) -> bool {
        if (!mbar_wait(&sm.staged, j & 1)) {
          report(p.status, kTimeoutSoftmax);
          return false;
        }
        const int ci = c0 + j;
        if (p.chunks[2 * ci + 1] == CH) {
          tma_store_3d(&tout, sm.buf[j % 3].w, 0, h, p.chunks[2 * ci]);
          bulk_commit();
          bulk_wait_read<0>();
        }
        return true;
      };
      constexpr uint32_t idesc64 = idesc_bf16(128, 64, false, false);
      constexpr uint32_t idesc_s = idesc_bf16(128, 128, false, true);
      for (int i = 0; i < total && i < 3; ++i) load(i);
      for (int i = 0; i < total; ++i) {
        if (!mbar_wait(&sm.conv_s, i & 1)) {
          report(p.status, kTimeoutSoftmax);
          break;
        }
        if (!mbar_wait(&sm.full[i % 3], (i / 3) & 1)) {
          report(p.status, kTimeoutFull);
          break;
        }
        tc_fence_after();
        const ChainBuf& b = sm.buf[i % 3];
        const uint32_t w0 = smem_u32(b.w), q0 = smem_u32(b.qg), k0 = smem_u32(b.kn), p0 = smem_u32(b.p);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)  // U^T = S0^T (-W)^T
          mma_f16_ts(tmem + 256, tmem + 384 + kk * 8, desc_sw128(w0 + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024),
                     idesc64, kk > 0);
        mma_commit(&sm.mma_u);
        if (!mbar_wait(&sm.conv_u, i & 1)) {
          report(p.status, kTimeoutSoftmax);
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < CH / 16; ++kk)  // S^T += Us^T K
          mma_f16_ts(tmem + 0, tmem + 480 + kk * 8, desc_sw128(k0 + kk * 2048, 8192, 1024), idesc_s, 1u);
        mma_commit(&sm.mma_s);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)  // O^T = S0^T (diag(γ) Q)^T
          mma_f16_ts(tmem + 320, tmem + 384 + kk * 8, desc_sw128(q0 + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024),
                     idesc64, kk > 0);
#pragma unroll
        for (int kk = 0; kk < CH / 16; ++kk)  // O^T += U^T P^T
          mma_f16_ts(tmem + 320, tmem + 448 + kk * 8, desc_sw128(p0 + kk * 32, 16, 1024), idesc64, 1u);
        mma_commit(&sm.mma_o);
        // chunk i-1's O, staged in its buffer, leaves by TMA store (whole chunks); then the
        // buffer takes chunk i+2
        if (i >= 1) {
          if (!store_staged(i - 1)) break;
          if (i + 2 < total) load(i + 2);
        }
      }
      if (total > 0) store_staged(total - 1);
      bulk_wait_all();
    }
  } else {
    const int c = threadIdx.x;  // value column = TMEM lane
    const uint32_t lb = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t t_s = tmem + lb, t_f = tmem + lb + 128, t_u = tmem + lb + 256, t_o = tmem + lb + 320;
    const uint32_t t_s0 = tmem + lb + 384, t_ub = tmem + lb + 448, t_us = tmem + lb + 480;
    const int64_t head_off = static_cast<int64_t>(h) * DK * DK;
    const float* init_head =
        sg.init_slot >= 0 ? p.state_pool + static_cast<int64_t>(sg.init_slot) * p.slot_stride + head_off : nullptr;
    bool ok = true;
    // 32 consecutive keys [32 j, 32 j + 32) of row c of the state S^T, from ``src``
    auto state_piece = [&](uint32_t (&x)[32], int src, int j) {
      if (src == kSrcTmemS || src == kSrcTmemF) {
        tmem_ld32((src == kSrcTmemS ? t_s : t_f) + 32 * j, x);
        tmem_wait_ld_regs(x);
      } else if (src == kSrcPool) {
#pragma unroll
        for (int e = 0; e < 32; ++e) x[e] = __float_as_uint(init_head[(32 * j + e) * DK + c]);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) x[e] = 0u;
      }
    };
    // O of chunk i (this thread's column c, read from TMEM) -> the chunk's -W slot (its data is
    // dead), transposed to rows [64 t][128 c]: a whole chunk then leaves by one TMA store from
    // the MMA warp, a partial one by 16-byte row pieces from these warps.
    auto load_o = [&](uint32_t (&ob)[32]) {  // bf16 pairs (t, t + 1)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t o[32];
        tmem_ld32(t_o + 32 * half, o);
        tmem_wait_ld_regs(o);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ob[16 * half + e] = pack_bf16(__uint_as_float(o[2 * e]), __uint_as_float(o[2 * e + 1]));
      }
    };
    auto stage_o = [&](int i, const uint32_t (&ob)[32]) {
      const int ci = c0 + i, row0 = p.chunks[2 * ci], nt = p.chunks[2 * ci + 1];
      uint16_t* stg = reinterpret_cast<uint16_t*>(sm.buf[i % 3].w);  // [64 t][128 c] bf16
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        stg[(2 * e) * DK + c] = static_cast<uint16_t>(ob[e] & 0xffffu);
        stg[(2 * e + 1) * DK + c] = static_cast<uint16_t>(ob[e] >> 16);
      }
      if (nt < CH) {
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four converting warps
        for (int e = c; e < nt * (DK / 8); e += 128) {
          const int t = e >> 4, u = e & 15;
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(row0 + t) * p.ld_out + h * DK + 8 * u) =
              *reinterpret_cast<const uint4*>(stg + static_cast<int>(t * DK + 8 * u));
        }
      } else {
        fence_proxy_async();  // these writes before the TMA store reads them
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.staged);
    };
    // the state (from ``src``) -> pool slot ``slot`` (layout [k][c] per head)
    auto save = [&](int src, int slot) {
      float* dst = p.state_pool + static_cast<int64_t>(slot) * p.slot_stride + head_off;
      for (int j = 0; j < 4; ++j) {
        uint32_t x[32];
        state_piece(x, src, j);
#pragma unroll
        for (int e = 0; e < 32; ++e) dst[(32 * j + e) * DK + c] = __uint_as_float(x[e]);
      }
    };
    int i = 0, cur = init_head ? kSrcPool : kSrcZero;
    for (int ri = 0; ri < n_runs && ok; ++ri) {
      const int nch = (run_len(ri) + CH - 1) / CH;
      const int run_src = ri >= 2 ? kSrcTmemF : cur;
      for (int t = 0; t < nch; ++t, ++i) {
        const int src = t == 0 ? run_src : kSrcTmemS;
        if (i > 0 && !mbar_wait(&sm.mma_s, (i - 1) & 1)) {
          report(p.status, kTimeoutMma);
          ok = false;
          break;
        }
        if (!mbar_wait(&sm.full[i % 3], (i / 3) & 1)) {
          report(p.status, kTimeoutFull);
          ok = false;
          break;
        }
        tc_fence_after();
        const ChainBuf& b = sm.buf[i % 3];
        // the chunk's start state: bf16 copy for the products, S^T scaled by γ_C for the update
        const float ec = b.ec[0];
        uint32_t s0[64];
        {
          uint32_t x[4][32];
          if (src == kSrcTmemS || src == kSrcTmemF) {  // four loads in flight, one wait
            const uint32_t from = src == kSrcTmemS ? t_s : t_f;
#pragma unroll
            for (int j = 0; j < 4; ++j) tmem_ld32(from + 32 * j, x[j]);
#pragma unroll
            for (int j = 0; j < 4; ++j) tmem_wait_ld_regs(x[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) state_piece(x[j], src, j);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              s0[16 * j + e] = pack_bf16(__uint_as_float(x[j][2 * e]), __uint_as_float(x[j][2 * e + 1]));
#pragma unroll
            for (int e = 0; e < 32; ++e) x[j][e] = __float_as_uint(__uint_as_float(x[j][e]) * ec);
            tmem_st32(t_s + 32 * j, x[j]);
          }
        }
        if (i > 0 && !mbar_wait(&sm.mma_o, (i - 1) & 1)) {  // the previous O^T no longer reads S0^T
          report(p.status, kTimeoutMma);
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 4; ++j) tmem_st16(t_s0 + 16 * j, *reinterpret_cast<uint32_t(*)[16]>(s0 + 16 * j));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.conv_s);
        uint32_t ov[32];  // the previous chunk's O (complete: its mma_o was waited for above)
        if (i > 0) load_o(ov);
        if (!mbar_wait(&sm.mma_u, i & 1)) {
          report(p.status, kTimeoutMma);
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // U = T'V + U^T, bf16; Us = e^{Γ_C-Γ_t} U, bf16
          uint32_t u[32], ub[16], us[16];
          tmem_ld32(t_u + 32 * half, u);
          tmem_wait_ld_regs(u);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int t = 32 * half + 4 * q;
            const float4 w4 = *reinterpret_cast<const float4*>(&b.ws[t]);
            const float a0 = __bfloat162float(b.tv[t * LDW + c]) + __uint_as_float(u[4 * q]);
            const float a1 = __bfloat162float(b.tv[(t + 1) * LDW + c]) + __uint_as_float(u[4 * q + 1]);
            const float a2 = __bfloat162float(b.tv[(t + 2) * LDW + c]) + __uint_as_float(u[4 * q + 2]);
            const float a3 = __bfloat162float(b.tv[(t + 3) * LDW + c]) + __uint_as_float(u[4 * q + 3]);
            ub[2 * q] = pack_bf16(a0, a1);
            ub[2 * q + 1] = pack_bf16(a2, a3);
            us[2 * q] = pack_bf16(a0 * w4.x, a1 * w4.y);
            us[2 * q + 1] = pack_bf16(a2 * w4.z, a3 * w4.w);
          }
          tmem_st16(t_ub + 16 * half, ub);
          tmem_st16(t_us + 16 * half, us);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.conv_u);
        if (i > 0) stage_o(i - 1, ov);
        cur = kSrcTmemS;
      }
      if (!ok) break;
      const bool fork = ri == 1 && sg.n_branches > 0;
      if ((ri == 0 && sg.save_slot >= 0) || fork) {
        if (cur == kSrcTmemS && !mbar_wait(&sm.mma_s, (i - 1) & 1)) {  // the run's last state update
          report(p.status, kTimeoutMma);
          ok = false;
          break;
        }
        tc_fence_after();
        if (ri == 0) save(cur, sg.save_slot);  // state after the cached prefix -> the pool slot
        if (fork) {                            // the trunk's final state, every branch's start
#pragma unroll 1
          for (int j = 0; j < 4; ++j) {
            uint32_t x[32];
            state_piece(x, cur, j);
            tmem_st32(t_f + 32 * j, x);
          }
          tmem_wait_st();
        }
      }
    }
    if (ok && i > 0) {
      if (mbar_wait(&sm.mma_o, (i - 1) & 1)) {
        tc_fence_after();
        uint32_t ov[32];
        load_o(ov);
        stage_o(i - 1, ov);
      } else {
        report(p.status, kTimeoutMma);
      }
    }
    tc_fence_before();
  }
  __syncwarp();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// y = bf16(bf16(w * bf16(x_hat)) * silu(z)) per (row, head) over dv (gated_rms_norm, fused.py:51-56).
__global__ void gated_rms_norm_kernel(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* z, int64_t ldz,
                                      const __nv_bfloat16* w, float eps, __nv_bfloat16* y, int64_t ldy, int rows,
                                      int heads, int dv) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows * heads) return;
  const int r = gw / heads, h = gw % heads;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(r) * ldx + h * dv;
  const __nv_bfloat16* zr = z + static_cast<int64_t>(r) * ldz + h * dv;
  __nv_bfloat16* yr = y + static_cast<int64_t>(r) * ldy + h * dv;
  float ss = 0.f;
  for (int c = lane; c < dv; c += 32) {
    const float f = __bfloat162float(xr[c]);
    ss += f * f;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / dv + eps);
  for (int c = lane; c < dv; c += 32) {
    const float t = bf16_round(__bfloat162float(w[c]) * bf16_round(__bfloat162float(xr[c]) * inv));
    yr[c] = __float2bfloat16_rn(t * silu(__bfloat162float(zr[c])));
  }
}

// Vector form for dv = 4 V (V = 1, 2): lane l holds elements [4 V l, 4 V l + 4 V) of its (row,
// head) in registers from one 8 V-byte load of x and of z, so x is read once. A warp takes
// ITEMS consecutive (row, head) items and issues all their loads before the first reduction,
// so each warp keeps ITEMS x 16 V bytes per lane in flight (the SiLU's exponential and
// reciprocal then overlap other warps' loads).
template <int V, int ITEMS>
__global__ void __launch_bounds__(256) gated_rms_norm_vec_kernel(const __nv_bfloat16* x, int64_t ldx,
                                                                 const __nv_bfloat16* z, int64_t ldz,
                                                                 const __nv_bfloat16* w, float eps, __nv_bfloat16* y,
                                                                 int64_t ldy, int rows, int heads) {
  using Vec = typename std::conditional<V == 1, uint2, uint4>::type;
  constexpr int E = 4 * V, DV = 32 * E;
  const int64_t total = static_cast<int64_t>(rows) * heads;
  const int64_t gw0 = ((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * ITEMS;
  const int lane = threadIdx.x & 31;
  if (gw0 >= total) return;
  const Vec wv = *reinterpret_cast<const Vec*>(w + lane * E);
  Vec xv[ITEMS], zv[ITEMS];
  int64_t yoff[ITEMS];
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const int64_t gw = gw0 + k < total ? gw0 + k : total - 1;
    const int64_t r = gw / heads, h = gw - r * heads;
    const int64_t off = h * DV + lane * E;
    xv[k] = *reinterpret_cast<const Vec*>(x + r * ldx + off);
    zv[k] = *reinterpret_cast<const Vec*>(z + r * ldz + off);
    yoff[k] = r * ldy + off;
  }
  const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv[k]);
    const __nv_bfloat16* ze = reinterpret_cast<const __nv_bfloat16*>(&zv[k]);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float f = __bfloat162float(xe[i]);
      ss += f * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / DV + eps);
    Vec yv;
    __nv_bfloat16* ye = reinterpret_cast<__nv_bfloat16*>(&yv);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float t = bf16_round(__bfloat162float(we[i]) * bf16_round(__bfloat162float(xe[i]) * inv));
      ye[i] = __float2bfloat16_rn(t * silu(__bfloat162float(ze[i])));
    }
    if (gw0 + k < total) *reinterpret_cast<Vec*>(y + yoff[k]) = yv;
  }
}

}  // namespace delta
}  // namespace dan

using namespace dan;

DAN_API int dan_causal_conv(const void* src, int64_t ld_src, const void* hist, int64_t ld_hist, const void* weight,
                            const int* prev, void* out, int64_t ld_out, int rows, int channels, void* stream) {
  DAN_REQUIRE(channels % 8 == 0 && ld_src % 8 == 0 && ld_out % 8 == 0 && (!hist || ld_hist % 8 == 0),
              "causal_conv: channels and strides must be multiples of 8");
  if (!rows) return 0;
  const dim3 grid((rows + delta::CONV_ROWS - 1) / delta::CONV_ROWS, (channels / delta::CONV_CPT + 255) / 256);
  delta::causal_conv_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), ld_src, static_cast<const __nv_bfloat16*>(hist), ld_hist,
      static_cast<const __nv_bfloat16*>(weight), prev, static_cast<__nv_bfloat16*>(out), ld_out, rows, channels);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_gather_rows(const void* src, int64_t ld_src, const void* hist, int64_t ld_hist, const int* codes,
                            int count, void* dst, int64_t ld_dst, int cols, void* stream) {
  DAN_REQUIRE(cols % 8 == 0 && ld_src % 8 == 0 && ld_dst % 8 == 0, "gather_rows: cols/strides must be multiples of 8");
  if (!count) return 0;
  delta::gather_rows_kernel<<<count, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), ld_src, static_cast<const __nv_bfloat16*>(hist), ld_hist, codes,
      static_cast<__nv_bfloat16*>(dst), ld_dst, cols);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int64_t dan_gated_delta_scratch_bytes(int n_chunks, int hk, int hv) {
  return static_cast<int64_t>(n_chunks) * (hv * delta::REC_V + hk * delta::REC_K);
}

// A second stream per device for the split launch below, created on first use and kept for
// the life of the process.
static cudaError_t side_stream(cudaStream_t* out) {
  static std::mutex mu;
  static cudaStream_t streams[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!streams[dev]) {
    e = cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking);
    if (e != cudaSuccess) return e;
  }
  *out = streams[dev];
  return cudaSuccess;
}

// Checks and launches of the two scan kernels: the pre-pass over the chunks, then the chains.
// With ``lead_chunks`` > 0 (the caller's estimate that the leading segment's chain outlasts the
// rest of the pre-pass; its chunks are [lead_chunk0, lead_chunk0 + lead_chunks)), the launch is
// split so that chain starts as soon as its own chunks are prepared, while the pre-pass of the
// other segments runs beside it on a second stream:
//   stream: prep(lead chunks) -> event A -> chain(segment 0) ---------------------> wait S
//   side:                        wait A -> prep(the other chunks) -> chains(other segments) -> event S
// The leading chain follows its pre-pass in stream order, so its CTAs (one SM each: their shared
// memory fills it) are placed on the SMs the pre-pass leaves empty before the other pre-pass
// CTAs, which wait for the event, fill the rest. Every kernel sees exactly the data it would in
// the unsplit order (a chain reads only its own segment's chunk records, and the records of
// different chunks are disjoint), so results are bit-identical; work queued on ``stream`` after
// the call waits for both streams' kernels.
static int scan_launch(const delta::ScanParams& p0, int n_segs, int dk, int dv, int64_t scratch_bytes,
                       int lead_chunk0, int lead_chunks, void* stream) {
  delta::ScanParams p = p0;
  DAN_REQUIRE(dk == delta::DK && dv == delta::DK, "gated_delta_scan: needs dk = dv = 128 (got %d, %d)", dk, dv);
  DAN_REQUIRE(p.ld_qkv % 8 == 0 && p.ld_out % 8 == 0, "gated_delta_scan: strides must be multiples of 8");
  DAN_REQUIRE(reinterpret_cast<uintptr_t>(p.q) % 16 == 0 && reinterpret_cast<uintptr_t>(p.k) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(p.v) % 16 == 0,
              "gated_delta_scan: q, k, v must be 16-byte aligned (their rows are bulk-copied)");
  DAN_REQUIRE(p.hk > 0 && p.hv % p.hk == 0, "gated_delta_scan: %d value heads not a multiple of %d key heads", p.hv,
              p.hk);
  DAN_REQUIRE(n_segs < 65536 && p.n_chunks < (1 << 30), "gated_delta_scan: too many segments or chunks");
  DAN_REQUIRE(scratch_bytes >= dan_gated_delta_scratch_bytes(p.n_chunks, p.hk, p.hv) &&
                  reinterpret_cast<uintptr_t>(p.scratch) % 16 == 0,
              "gated_delta_scan: scratch needs %lld bytes, 16-byte aligned (got %lld)",
              static_cast<long long>(dan_gated_delta_scratch_bytes(p.n_chunks, p.hk, p.hv)),
              static_cast<long long>(scratch_bytes));
  DAN_REQUIRE(lead_chunks == 0 || (lead_chunk0 >= 0 && lead_chunks > 0 && lead_chunk0 + lead_chunks <= p.n_chunks),
              "gated_delta_scan: lead chunks [%d, %d) outside the %d chunks", lead_chunk0, lead_chunk0 + lead_chunks,
              p.n_chunks);
  if (!n_segs || !p.n_chunks) return 0;
  static std::atomic<uint64_t> prep_conf{0}, state_conf{0};
  DAN_CUDA(smem_limit_once(delta::chunk_prep_kernel, static_cast<int>(sizeof(delta::PrepSmem)), prep_conf));
  DAN_CUDA(smem_limit_once(delta::chunk_state_kernel, delta::CHAIN_SMEM, state_conf));
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // O of whole chunks by TMA store: [rows][hv][128] bf16, box one head x 64 rows, no swizzle (the
  // rows the kernel stores always exist; the row extent only bounds the map)
  CUtensorMap tout;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(delta::DK), static_cast<uint64_t>(p.hv), uint64_t{1} << 24};
    const uint64_t strides[2] = {static_cast<uint64_t>(delta::DK) * 2, static_cast<uint64_t>(p.ld_out) * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(delta::DK), 1, static_cast<uint32_t>(delta::CH)};
    int rc = make_tmap(&tout, p.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  const size_t prep_smem = sizeof(delta::PrepSmem);
  if (lead_chunks == 0 || lead_chunks == p.n_chunks || n_segs < 2) {
    delta::chunk_prep_kernel<<<dim3(p.n_chunks, p.hv), 256, prep_smem, st>>>(p);
    DAN_CUDA(cudaGetLastError());
    delta::chunk_state_kernel<<<dim3(p.hv, n_segs), 160, delta::CHAIN_SMEM, st>>>(tout, p);
    DAN_CUDA(cudaGetLastError());
    return 0;
  }
  cudaStream_t side = nullptr;
  DAN_CUDA(side_stream(&side));
  cudaEvent_t ev_a = nullptr, ev_s = nullptr;
  DAN_CUDA(cudaEventCreateWithFlags(&ev_a, cudaEventDisableTiming));
  cudaError_t e = cudaEventCreateWithFlags(&ev_s, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    cudaEventDestroy(ev_a);
    return ::dan::fail(-5, "cudaEventCreateWithFlags failed: %s", cudaGetErrorString(e));
  }
  delta::ScanParams pa = p, pb = p, ps = p;
  pa.chunk_base = lead_chunk0;                                // the leading segment's chunks
  pb.skip_at = lead_chunk0, pb.skip_len = lead_chunks;        // every other chunk
  ps.seg_base = 1;                                            // segments 1 .. n_segs - 1
  delta::chunk_prep_kernel<<<dim3(lead_chunks, p.hv), 256, prep_smem, st>>>(pa);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaEventRecord(ev_a, st);
  if (e == cudaSuccess) {
    delta::chunk_state_kernel<<<dim3(p.hv, 1), 160, delta::CHAIN_SMEM, st>>>(tout, p);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamWaitEvent(side, ev_a, 0);
  if (e == cudaSuccess) {
    delta::chunk_prep_kernel<<<dim3(p.n_chunks - lead_chunks, p.hv), 256, prep_smem, side>>>(pb);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    delta::chunk_state_kernel<<<dim3(p.hv, n_segs - 1), 160, delta::CHAIN_SMEM, side>>>(tout, ps);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaEventRecord(ev_s, side);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, ev_s, 0);
  cudaEventDestroy(ev_a);  // released once the work that records or waits on them has run
  cudaEventDestroy(ev_s);
  if (e != cudaSuccess) return ::dan::fail(-5, "gated_delta_scan split launch failed: %s", cudaGetErrorString(e));
  return 0;
}

static delta::ScanParams scan_params(const void* q, const void* k, const void* v, int64_t ld_qkv, const int* segs,
                                     const int* branches, const int* chunks, int n_chunks, float* state_pool,
                                     int64_t slot_stride, void* out, int64_t ld_out, int hk, int hv, float q_scale,
                                     void* scratch, int32_t* status) {
  delta::ScanParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.ld_qkv = ld_qkv;
  p.segs = reinterpret_cast<const delta::Seg*>(segs);
  p.branches = branches;
  p.state_pool = state_pool;
  p.slot_stride = slot_stride;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.hk = hk;
  p.hv = hv;
  p.q_scale = q_scale;
  p.chunks = chunks;
  p.n_chunks = n_chunks;
  p.scratch = static_cast<uint8_t*>(scratch);
  p.status = status;
  return p;
}

DAN_API int dan_gated_delta_scan(const void* q, const void* k, const void* v, int64_t ld_qkv, const void* b,
                                 const void* a, int64_t ld_ba, const float* a_log, const float* dt_bias,
                                 const int* segs, int n_segs, const int* branches, const int* chunks, int n_chunks,
                                 float* state_pool, int64_t slot_stride, void* out, int64_t ld_out, int hk, int hv,
                                 int dk, int dv, float q_scale, void* scratch, int64_t scratch_bytes, int lead_chunk0,
                                 int lead_chunks, int32_t* status, void* stream) {
  DAN_REQUIRE(a_log != nullptr && dt_bias != nullptr, "gated_delta_scan: A_log and dt_bias are required");
  delta::ScanParams p = scan_params(q, k, v, ld_qkv, segs, branches, chunks, n_chunks, state_pool, slot_stride, out,
                                    ld_out, hk, hv, q_scale, scratch, status);
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.ld_ba = ld_ba;
  p.a_log = a_log;
  p.dt_bias = dt_bias;
  return scan_launch(p, n_segs, dk, dv, scratch_bytes, lead_chunk0, lead_chunks, stream);
}

DAN_API int dan_delta_rule_scan(const void* q, const void* k, const void* v, int64_t ld_qkv, const void* beta,
                                int64_t ld_beta, const float* g, int64_t ld_g, const int* segs, int n_segs,
                                const int* branches, const int* chunks, int n_chunks, float* state_pool,
                                int64_t slot_stride, void* out, int64_t ld_out, int hk, int hv, int dk, int dv,
                                float q_scale, void* scratch, int64_t scratch_bytes, int32_t* status, void* stream) {
  DAN_REQUIRE(beta != nullptr && g != nullptr, "delta_rule_scan: beta and g are required");
  delta::ScanParams p = scan_params(q, k, v, ld_qkv, segs, branches, chunks, n_chunks, state_pool, slot_stride, out,
                                    ld_out, hk, hv, q_scale, scratch, status);
  p.b = static_cast<const __nv_bfloat16*>(beta);
  p.ld_ba = ld_beta;
  p.g_given = g;
  p.ld_g = ld_g;
  return scan_launch(p, n_segs, dk, dv, scratch_bytes, 0, 0, stream);
}

DAN_API int dan_gated_rms_norm(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* w, float eps,
                               void* y, int64_t ldy, int rows, int heads, int dv, void* stream) {
  if (!rows) return 0;
  const int64_t warps = static_cast<int64_t>(rows) * heads;
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if ((dv == 128 || dv == 256) && a16(x) && a16(z) && a16(w) && a16(y) && ldx % 8 == 0 && ldz % 8 == 0 &&
      ldy % 8 == 0) {
    constexpr int kItems128 = delta::GNORM_ITEMS, kItems256 = kItems128 > 1 ? kItems128 / 2 : 1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dv == 128)
      delta::gated_rms_norm_vec_kernel<1, kItems128><<<static_cast<unsigned>((warps + 8 * kItems128 - 1) /
                                                                             (8 * kItems128)), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(z), ldz,
          static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(y), ldy, rows, heads);
    else
      delta::gated_rms_norm_vec_kernel<2, kItems256><<<static_cast<unsigned>((warps + 8 * kItems256 - 1) /
                                                                             (8 * kItems256)), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(z), ldz,
          static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(y), ldy, rows, heads);
    DAN_CUDA(cudaGetLastError());
    return 0;
  }
  delta::gated_rms_norm_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0,
                                 static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(z), ldz,
      static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(y), ldy, rows, heads, dv);
  DAN_CUDA(cudaGetLastError());
  return 0;
}
