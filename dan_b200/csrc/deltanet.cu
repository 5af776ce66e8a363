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
// k-1 rows as conv history. The scan kernel keeps one head's 128 x 128 state
// in registers (fp32) across the whole segment: it walks the trunk in chunks
// of 64 tokens, writes the state at the prefix-save cut to the pool, keeps the
// trunk's final state as a second register copy and forks each branch from it:
// the state never round-trips to HBM.
//
// Recurrence per token (delta_rule_torch, qwen3_5.py:103-133):
//   a = exp(g);  S <- a S;  u = beta (v - S^T k);  S <- S + k u^T;  o = S^T q
// with k, q l2-normalised (eps 1e-6) and q scaled by Dk^-0.5; evaluated per
// chunk in the WY form on the tensor cores (see chunk_scan_kernel).
#include "common.cuh"

namespace dan {
namespace delta {

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
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
__global__ void causal_conv_kernel(const __nv_bfloat16* src, int64_t ld_src, const __nv_bfloat16* hist,
                                   int64_t ld_hist, const __nv_bfloat16* w, const int* prev, __nv_bfloat16* out,
                                   int64_t ld_out, int rows, int channels) {
  const int r = blockIdx.x;
  const int* pr = prev + 3 * r;
  const __nv_bfloat16* rows4[4] = {code_row(pr[2], src, ld_src, hist, ld_hist),
                                   code_row(pr[1], src, ld_src, hist, ld_hist),
                                   code_row(pr[0], src, ld_src, hist, ld_hist), src + static_cast<int64_t>(r) * ld_src};
  for (int c0 = threadIdx.x * 8; c0 < channels; c0 += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // weights [C, 4]: 8 channels x 4 taps = 32 bf16 = 4 x 16 B
    uint4 wv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) wv[i] = reinterpret_cast<const uint4*>(w + static_cast<int64_t>(c0) * 4)[i];
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(wv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!rows4[j]) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(rows4[j] + c0);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[t] += __bfloat162float(we[t * 4 + j]) * __bfloat162float(e[t]);
    }
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int t = 0; t < 4; ++t) op[t] = pack_bf16(silu(acc[2 * t]), silu(acc[2 * t + 1]));
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(r) * ld_out + c0) = o;
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

// Segment record (int32 x 8): trunk_start, trunk_len, cut, init_slot, save_slot, branch0, n_branches, 0.
// Branch record (int32 x 2): start, len.
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
  const float* a_log;    // [hv]
  const float* dt_bias;  // [hv]
  const Seg* segs;
  const int* branches;
  float* state_pool;  // [slots, hv, dk, dv] of this layer (slot stride given)
  int64_t slot_stride;
  __nv_bfloat16* out;  // [rows, hv, dv]
  int64_t ld_out;
  int hk, hv;
  float q_scale;
};

constexpr int DK = 128;

// ---------------------------------------------------------------------------------
// Chunked gated delta rule on the tensor cores (mma.sync m16n8k16, bf16 operands, fp32
// accumulation). One CTA of 8 warps per (value head, segment) walks the segment's runs in
// chunks of CH = 64 tokens. With Γ_t the cumulative log decay inside a chunk (γ_t = e^Γ_t),
// the token recurrence S_t = d_t S_{t-1} + k_t u_t^T, u_t = β_t (v_t - k_t^T d_t S_{t-1}),
// o_t = q_t^T S_t unrolls over a chunk that starts from state S0 to
//   A  = strictly_lower(β_t e^{Γ_t-Γ_s} k_t.k_s),  T = (I + A)^-1,  T' = T diag(β)
//   U  = T' V - (T' diag(γ) K) S0                       (the chunk's u_t)
//   O  = diag(γ) Q S0 + (e^{Γ_t-Γ_s} q_t.k_s, s <= t) U
//   S  = γ_C S0 + K^T diag(e^{Γ_C-Γ_t}) U
// (the WY form of the delta rule; every decay factor is e^{difference} <= 1). The state
// lives in registers in fp32 (warp w: rows [16w, 16w+16) of S, all 128 columns); a bf16
// copy in shared memory is the operand of the S0 products. T is solved in fp32: 16x16
// diagonal blocks by substitution, then two levels of block merges.
constexpr int CH = 64;
constexpr int LDW = DK + 8;  // bf16 row stride of 128-wide tiles: 272 B, ldmatrix rows on distinct banks
constexpr int LDN = CH + 8;  // bf16 row stride of 64-wide tiles
constexpr int LDF = CH + 4;  // fp32 row stride of 64 x 64 tiles

struct ChunkSmem {
  __nv_bfloat16 qn[CH * LDW];  // l2-normalised, scaled q
  __nv_bfloat16 kn[CH * LDW];  // l2-normalised k
  __nv_bfloat16 v[CH * LDW];
  __nv_bfloat16 kg[CH * LDW];  // γ_t k_t, then -W
  __nv_bfloat16 u[CH * LDW];   // U
  __nv_bfloat16 us[CH * LDW];  // e^{Γ_C-Γ_t} U (fp32 scratch of the block merges before that)
  __nv_bfloat16 s0[DK * LDW];  // chunk-start state, bf16
  float a[CH * LDF];           // A
  float tf[CH * LDF];          // T = (I + A)^-1
  __nv_bfloat16 tb[CH * LDN];  // T diag(β)
  __nv_bfloat16 pb[CH * LDN];  // e^{Γ_t-Γ_s} q_t.k_s (s <= t)
  float gam[CH], eg[CH], beta[CH], graw[CH];
};

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

// One chunk of a run: rows [row0, row0 + nt) of the packed batch, state S in and out.
__device__ __forceinline__ void scan_chunk(const ScanParams& p, ChunkSmem& sm, float (&S)[16][4], int h, int kh,
                                           float a_neg, float dtb, int row0, int nt) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  // ---- stage: q, k (l2-normalised), v, gates; S0 as bf16; T cleared
  {
    if (lane < 8) {
      const int t = warp * 8 + lane;
      float bb = 0.f, gg = 0.f;
      if (t < nt) {
        const int64_t row = row0 + t;
        bb = 1.f / (1.f + __expf(-__bfloat162float(p.b[row * p.ld_ba + h])));
        gg = a_neg * softplus(__bfloat162float(p.a[row * p.ld_ba + h]) + dtb);
      }
      sm.beta[t] = bb;
      sm.graw[t] = gg;
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint2 qw[4], kw[4], vw[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // the four rows' loads issued before any is used
        const int64_t row = row0 + min(warp * 8 + half * 4 + i, nt - 1);
        qw[i] = __ldg(reinterpret_cast<const uint2*>(p.q + row * p.ld_qkv + kh * DK + lane * 4));
        kw[i] = __ldg(reinterpret_cast<const uint2*>(p.k + row * p.ld_qkv + kh * DK + lane * 4));
        vw[i] = __ldg(reinterpret_cast<const uint2*>(p.v + row * p.ld_qkv + h * DK + lane * 4));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = warp * 8 + half * 4 + i;
        const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qw[i]);
        const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kw[i]);
        const float2 qa = __bfloat1622float2(q2[0]), qb = __bfloat1622float2(q2[1]);
        const float2 ka = __bfloat1622float2(k2[0]), kb = __bfloat1622float2(k2[1]);
        float sq = qa.x * qa.x + qa.y * qa.y + qb.x * qb.x + qb.y * qb.y;
        float sk = ka.x * ka.x + ka.y * ka.y + kb.x * kb.x + kb.y * kb.y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          sq += __shfl_xor_sync(0xffffffffu, sq, o);
          sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        const bool live = t < nt;
        const float nq = live ? rsqrtf(sq + 1e-6f) * p.q_scale : 0.f, nk = live ? rsqrtf(sk + 1e-6f) : 0.f;
        *reinterpret_cast<uint2*>(&sm.qn[t * LDW + lane * 4]) =
            make_uint2(pack_bf16(qa.x * nq, qa.y * nq), pack_bf16(qb.x * nq, qb.y * nq));
        *reinterpret_cast<uint2*>(&sm.kn[t * LDW + lane * 4]) =
            make_uint2(pack_bf16(ka.x * nk, ka.y * nk), pack_bf16(kb.x * nk, kb.y * nk));
        *reinterpret_cast<uint2*>(&sm.v[t * LDW + lane * 4]) = live ? vw[i] : make_uint2(0u, 0u);
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      st_bf2(&sm.s0[(16 * warp + g) * LDW + 8 * j + 2 * c], S[j][0], S[j][1]);
      st_bf2(&sm.s0[(16 * warp + g + 8) * LDW + 8 * j + 2 * c], S[j][2], S[j][3]);
    }
    for (int i = tid; i < CH * LDF; i += blockDim.x) sm.tf[i] = 0.f;
  }
  __syncthreads();
  if (warp == 0) {  // Γ: inclusive prefix sum of the log decays
    const float v0 = sm.graw[2 * lane], v1 = sm.graw[2 * lane + 1];
    float incl = v0 + v1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float g0 = incl - v1, g1 = incl;
    sm.gam[2 * lane] = g0;
    sm.gam[2 * lane + 1] = g1;
    sm.eg[2 * lane] = __expf(g0);
    sm.eg[2 * lane + 1] = __expf(g1);
  }
  __syncthreads();
  const float gc = sm.gam[nt - 1];
  for (int e = tid; e < CH * (DK / 8); e += blockDim.x) {  // kg = γ_t k_t, 8 elements at a time
    const int t = e >> 4, col = (e & 15) * 8;
    const float s = sm.eg[t];
    uint4 w = *reinterpret_cast<const uint4*>(&sm.kn[t * LDW + col]);
    __nv_bfloat162* w2 = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(w2[i]);
      w2[i] = __floats2bfloat162_rn(f.x * s, f.y * s);
    }
    *reinterpret_cast<uint4*>(&sm.kg[t * LDW + col]) = w;
  }
  // ---- K K^T -> A and Q K^T -> P (warp: rows [16 tm, +16), columns [32 sh, +32))
  {
    const int tm = warp & 3, sh = warp >> 2;
    float G[4][4] = {}, Pq[4][4] = {};
#pragma unroll 1
    for (int kk = 0; kk < DK / 16; ++kk) {
      uint32_t ak[4], aq[4];
      ldsm4(ak, a_rows(sm.kn, LDW, 16 * tm, 16 * kk, lane));
      ldsm4(aq, a_rows(sm.qn, LDW, 16 * tm, 16 * kk, lane));
#pragma unroll
      for (int np = 0; np < 2; ++np) {
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
  // ---- T = (I + A)^-1: diagonal 16 x 16 blocks by forward substitution (thread: one column)
  if (tid < 64) {
    const int d = tid >> 4, j = tid & 15;
    float x[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float acc = (t == j) ? 1.f : 0.f;
#pragma unroll
      for (int s = 0; s < t; ++s) acc -= sm.a[(16 * d + t) * LDF + 16 * d + s] * x[s];
      x[t] = acc;
      sm.tf[(16 * d + t) * LDF + 16 * d + j] = acc;
    }
  }
  __syncthreads();
  float* ysc = reinterpret_cast<float*>(sm.us);  // 32 x 33 fp32 scratch
  {  // level 1: T[d+1][d] = -T[d+1][d+1] A[d+1][d] T[d][d] for d = 0, 2
    const int q = tid >> 7, r = (tid >> 3) & 15, cc = (tid & 7) * 2, d = 2 * q;
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float av = sm.a[(16 * (d + 1) + r) * LDF + 16 * d + k];
      y0 += av * sm.tf[(16 * d + k) * LDF + 16 * d + cc];
      y1 += av * sm.tf[(16 * d + k) * LDF + 16 * d + cc + 1];
    }
    ysc[(q * 16 + r) * 33 + cc] = y0;
    ysc[(q * 16 + r) * 33 + cc + 1] = y1;
    __syncthreads();
    float x0 = 0.f, x1 = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float tv = sm.tf[(16 * (d + 1) + r) * LDF + 16 * (d + 1) + k];
      x0 -= tv * ysc[(q * 16 + k) * 33 + cc];
      x1 -= tv * ysc[(q * 16 + k) * 33 + cc + 1];
    }
    sm.tf[(16 * (d + 1) + r) * LDF + 16 * d + cc] = x0;
    sm.tf[(16 * (d + 1) + r) * LDF + 16 * d + cc + 1] = x1;
  }
  __syncthreads();
  {  // level 2: T[32:64][0:32] = -T[32:64][32:64] A[32:64][0:32] T[0:32][0:32]
    const int r = tid >> 3, cq = (tid & 7) * 4;
    float y[4] = {};
    for (int k = 0; k < 32; ++k) {
      const float av = sm.a[(32 + r) * LDF + k];
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] += av * sm.tf[k * LDF + cq + e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) ysc[r * 33 + cq + e] = y[e];
    __syncthreads();
    float x[4] = {};
    for (int k = 0; k < 32; ++k) {
      const float tv = sm.tf[(32 + r) * LDF + 32 + k];
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] -= tv * ysc[k * 33 + cq + e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) sm.tf[(32 + r) * LDF + cq + e] = x[e];
  }
  __syncthreads();
  for (int e = tid; e < CH * CH / 2; e += blockDim.x) {  // T' = T diag(β), bf16
    const int t = e >> 5, s = (e & 31) * 2;
    st_bf2(&sm.tb[t * LDN + s], sm.tf[t * LDF + s] * sm.beta[s], sm.tf[t * LDF + s + 1] * sm.beta[s + 1]);
  }
  __syncthreads();
  // ---- W = T' diag(γ) K  (warp: rows [16 tm, +16), columns [64 tn, +64))
  const int tm = warp & 3, tn = warp >> 2;
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll 1
  for (int kk = 0; kk < CH / 16; ++kk) {
    uint32_t a[4];
    ldsm4(a, a_rows(sm.tb, LDN, 16 * tm, 16 * kk, lane));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm4t(b, b_krows(sm.kg, LDW, 16 * kk, 64 * tn + 16 * np, lane));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
  __syncthreads();  // every warp is done reading kg: it now holds -W
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int t = 16 * tm + g, col = 64 * tn + 8 * j + 2 * c;
    st_bf2(&sm.kg[t * LDW + col], -acc[j][0], -acc[j][1]);
    st_bf2(&sm.kg[(t + 8) * LDW + col], -acc[j][2], -acc[j][3]);
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  }
  __syncthreads();
  // ---- U = T' V - W S0
#pragma unroll 1
  for (int kk = 0; kk < CH / 16; ++kk) {
    uint32_t a[4];
    ldsm4(a, a_rows(sm.tb, LDN, 16 * tm, 16 * kk, lane));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm4t(b, b_krows(sm.v, LDW, 16 * kk, 64 * tn + 16 * np, lane));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
#pragma unroll 1
  for (int kk = 0; kk < DK / 16; ++kk) {
    uint32_t a[4];
    ldsm4(a, a_rows(sm.kg, LDW, 16 * tm, 16 * kk, lane));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm4t(b, b_krows(sm.s0, LDW, 16 * kk, 64 * tn + 16 * np, lane));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
  {
    const int t = 16 * tm + g;
    const float w0 = __expf(gc - sm.gam[t]), w1 = __expf(gc - sm.gam[t + 8]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = 64 * tn + 8 * j + 2 * c;
      st_bf2(&sm.u[t * LDW + col], acc[j][0], acc[j][1]);
      st_bf2(&sm.u[(t + 8) * LDW + col], acc[j][2], acc[j][3]);
      st_bf2(&sm.us[t * LDW + col], acc[j][0] * w0, acc[j][1] * w0);
      st_bf2(&sm.us[(t + 8) * LDW + col], acc[j][2] * w1, acc[j][3] * w1);
      acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    }
  }
  __syncthreads();
  // ---- O = diag(γ) Q S0 + P U -> out rows
#pragma unroll 1
  for (int kk = 0; kk < DK / 16; ++kk) {
    uint32_t a[4];
    ldsm4(a, a_rows(sm.qn, LDW, 16 * tm, 16 * kk, lane));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm4t(b, b_krows(sm.s0, LDW, 16 * kk, 64 * tn + 16 * np, lane));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
  {
    const float e0 = sm.eg[16 * tm + g], e1 = sm.eg[16 * tm + g + 8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[j][0] *= e0;
      acc[j][1] *= e0;
      acc[j][2] *= e1;
      acc[j][3] *= e1;
    }
  }
#pragma unroll 1
  for (int kk = 0; kk < CH / 16; ++kk) {
    uint32_t a[4];
    ldsm4(a, a_rows(sm.pb, LDN, 16 * tm, 16 * kk, lane));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm4t(b, b_krows(sm.u, LDW, 16 * kk, 64 * tn + 16 * np, lane));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
  {
    const int t = 16 * tm + g;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = h * DK + 64 * tn + 8 * j + 2 * c;
      if (t < nt) st_bf2(p.out + static_cast<int64_t>(row0 + t) * p.ld_out + col, acc[j][0], acc[j][1]);
      if (t + 8 < nt) st_bf2(p.out + static_cast<int64_t>(row0 + t + 8) * p.ld_out + col, acc[j][2], acc[j][3]);
    }
  }
  // ---- S = γ_C S0 + K^T (e^{Γ_C - Γ_t} U)  (warp: rows [16 w, +16) of S)
  {
    const float ec = __expf(gc);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      S[j][0] *= ec;
      S[j][1] *= ec;
      S[j][2] *= ec;
      S[j][3] *= ec;
    }
#pragma unroll 1
    for (int kk = 0; kk < CH / 16; ++kk) {
      uint32_t a[4];
      ldsm4t(a, a_cols(sm.kn, LDW, 16 * warp, 16 * kk, lane));
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t b[4];
        ldsm4t(b, b_krows(sm.us, LDW, 16 * kk, 16 * np, lane));
        mma16816(S[2 * np], a, b[0], b[1]);
        mma16816(S[2 * np + 1], a, b[2], b[3]);
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void state_io(float (&S)[16][4], float* st, bool load) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float* r0 = st + (16 * warp + g) * DK + 8 * j + 2 * c;
    float* r1 = r0 + 8 * DK;
    if (load) {
      const float2 x = *reinterpret_cast<const float2*>(r0), y = *reinterpret_cast<const float2*>(r1);
      S[j][0] = x.x, S[j][1] = x.y, S[j][2] = y.x, S[j][3] = y.y;
    } else {
      *reinterpret_cast<float2*>(r0) = make_float2(S[j][0], S[j][1]);
      *reinterpret_cast<float2*>(r1) = make_float2(S[j][2], S[j][3]);
    }
  }
}

// One CTA: (value head blockIdx.x, segment blockIdx.y). Runs in order: trunk up to the save
// cut, trunk after it, then each branch from the trunk's final state (kept in registers).
__global__ void __launch_bounds__(256, 1) chunk_scan_kernel(ScanParams p) {
  extern __shared__ __align__(16) uint8_t dsm[];
  ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>(dsm);
  const int h = blockIdx.x;
  const Seg sg = p.segs[blockIdx.y];
  const int kh = h / (p.hv / p.hk);
  const float a_neg = -__expf(p.a_log[h]), dtb = p.dt_bias[h];
  float S[16][4], F[16][4];
  if (sg.init_slot >= 0) {
    state_io(S, p.state_pool + static_cast<int64_t>(sg.init_slot) * p.slot_stride + static_cast<int64_t>(h) * DK * DK,
             true);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.f;
  }
  const int n_runs = 2 + sg.n_branches;
  for (int ri = 0; ri < n_runs; ++ri) {
    int start, len;
    if (ri == 0) {
      start = sg.trunk_start;
      len = sg.cut;
    } else if (ri == 1) {
      start = sg.trunk_start + sg.cut;
      len = sg.trunk_len - sg.cut;
    } else {
      const int* br = p.branches + 2 * (sg.branch0 + ri - 2);
      start = br[0];
      len = br[1];
      if (ri > 2) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) S[j][e] = F[j][e];
      }
    }
    for (int t0 = 0; t0 < len; t0 += CH) scan_chunk(p, sm, S, h, kh, a_neg, dtb, start + t0, min(CH, len - t0));
    if (ri == 0 && sg.save_slot >= 0)  // state after the cached prefix -> the pool slot
      state_io(S, p.state_pool + static_cast<int64_t>(sg.save_slot) * p.slot_stride + static_cast<int64_t>(h) * DK * DK,
               false);
    if (ri == 1 && sg.n_branches > 1) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) F[j][e] = S[j][e];
    }
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

}  // namespace delta
}  // namespace dan

using namespace dan;

DAN_API int dan_causal_conv(const void* src, int64_t ld_src, const void* hist, int64_t ld_hist, const void* weight,
                            const int* prev, void* out, int64_t ld_out, int rows, int channels, void* stream) {
  DAN_REQUIRE(channels % 8 == 0 && ld_src % 8 == 0 && ld_out % 8 == 0 && (!hist || ld_hist % 8 == 0),
              "causal_conv: channels and strides must be multiples of 8");
  if (!rows) return 0;
  delta::causal_conv_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
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

DAN_API int dan_gated_delta_scan(const void* q, const void* k, const void* v, int64_t ld_qkv, const void* b,
                                 const void* a, int64_t ld_ba, const float* a_log, const float* dt_bias,
                                 const int* segs, int n_segs, const int* branches, float* state_pool,
                                 int64_t slot_stride, void* out, int64_t ld_out, int hk, int hv, int dk, int dv,
                                 float q_scale, void* stream) {
  DAN_REQUIRE(dk == delta::DK && dv == delta::DK, "gated_delta_scan: needs dk = dv = 128 (got %d, %d)", dk, dv);
  DAN_REQUIRE(ld_qkv % 8 == 0 && ld_out % 8 == 0, "gated_delta_scan: strides must be multiples of 8");
  DAN_REQUIRE(hk > 0 && hv % hk == 0, "gated_delta_scan: %d value heads not a multiple of %d key heads", hv, hk);
  DAN_REQUIRE(n_segs < 65536, "gated_delta_scan: too many segments");
  if (!n_segs) return 0;
  delta::ScanParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.ld_qkv = ld_qkv;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.ld_ba = ld_ba;
  p.a_log = a_log;
  p.dt_bias = dt_bias;
  p.segs = reinterpret_cast<const delta::Seg*>(segs);
  p.branches = branches;
  p.state_pool = state_pool;
  p.slot_stride = slot_stride;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.hk = hk;
  p.hv = hv;
  p.q_scale = q_scale;
  static bool configured = false;
  if (!configured) {
    DAN_CUDA(cudaFuncSetAttribute(delta::chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(sizeof(delta::ChunkSmem))));
    configured = true;
  }
  delta::chunk_scan_kernel<<<dim3(hv, n_segs), 256, sizeof(delta::ChunkSmem), static_cast<cudaStream_t>(stream)>>>(p);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_gated_rms_norm(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* w, float eps,
                               void* y, int64_t ldy, int rows, int heads, int dv, void* stream) {
  if (!rows) return 0;
  const int64_t warps = static_cast<int64_t>(rows) * heads;
  delta::gated_rms_norm_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0,
                                 static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(z), ldz,
      static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(y), ldy, rows, heads, dv);
  DAN_CUDA(cudaGetLastError());
  return 0;
}
