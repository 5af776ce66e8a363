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
// k-1 rows as conv history. The scan kernel keeps the state of 32 value
// columns of one head in registers (fp32), walks the trunk, writes the state at
// the prefix-save cut to the pool, parks the trunk's final state in shared
// memory and forks each branch from it: the state never round-trips to HBM.
//
// Recurrence per token (exactly the reference's chunked algebra unrolled):
//   a = exp(g);  S <- a S;  u = beta (v - S^T k);  S <- S + k u^T;  o = S^T q
// with k, q l2-normalised (eps 1e-6) and q scaled by Dk^-0.5, in fp32.
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

constexpr int DK = 128, COLS = 16, HALF = 64, TCHUNK = 16;
// Staged q / k rows are padded so the two lane halves (rows [0, 64) and [64, 128)) read
// different shared-memory banks: element r of a row sits at r + 4 * (r / 64).
constexpr int KPAD = DK + 8;
__device__ __forceinline__ int kidx(int r) { return r + ((r >> 6) << 2); }

// One warp: (segment, value head, 16-column block). Lanes 2j and 2j+1 own column j of the
// state, rows [0, 64) and [64, 128) of S[:, j]; their partial dot products meet in one shuffle.
__global__ void __launch_bounds__(32) gated_delta_scan_kernel(ScanParams p) {
  const int cb = blockIdx.x, h = blockIdx.y;
  const Seg sg = p.segs[blockIdx.z];
  const int lane = threadIdx.x;
  const int jj = lane >> 1, half = lane & 1, r0 = half * HALF;
  const int kh = h / (p.hv / p.hk);
  const int col = cb * COLS + jj;
  __shared__ __align__(16) float qs[TCHUNK][KPAD];
  __shared__ __align__(16) float ks[TCHUNK][KPAD];
  __shared__ float vs[TCHUNK][COLS];
  __shared__ float qk[TCHUNK], gs[TCHUNK], bs[TCHUNK];
  __shared__ float fork[DK][COLS + 1];

  const float a_log = -__expf(p.a_log[h]);
  const float dtb = p.dt_bias[h];
  float S[HALF];
  if (sg.init_slot >= 0) {
    const float* st = p.state_pool + static_cast<int64_t>(sg.init_slot) * p.slot_stride +
                      static_cast<int64_t>(h) * DK * DK + static_cast<int64_t>(r0) * DK + col;
#pragma unroll
    for (int i = 0; i < HALF; ++i) S[i] = st[static_cast<int64_t>(i) * DK];
  } else {
#pragma unroll
    for (int i = 0; i < HALF; ++i) S[i] = 0.f;
  }

  // Runs in order: trunk up to the save cut, trunk after it, then each branch from the
  // trunk's final state (parked in shared memory).
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
        for (int i = 0; i < HALF; ++i) S[i] = fork[r0 + i][jj];
      }
    }
    for (int t0 = 0; t0 < len; t0 += TCHUNK) {
      const int nt = min(TCHUNK, len - t0);
      __syncwarp();
      // Stage the chunk with every load issued up front (one memory latency per chunk):
      // q and k (4 elements per lane per token), this lane's v column, and the gates
      // (lane t handles token t).
      uint2 qw[TCHUNK], kw[TCHUNK];
      float vr[TCHUNK];
#pragma unroll
      for (int t = 0; t < TCHUNK; ++t) {  // unconditional (tail rows clamped) so all loads issue at once
        const int64_t row = start + t0 + min(t, nt - 1);
        qw[t] = __ldg(reinterpret_cast<const uint2*>(p.q + row * p.ld_qkv + kh * DK + lane * 4));
        kw[t] = __ldg(reinterpret_cast<const uint2*>(p.k + row * p.ld_qkv + kh * DK + lane * 4));
        vr[t] = __bfloat162float(__ldg(p.v + row * p.ld_qkv + h * DK + col));
      }
      if (lane < nt) {
        const int64_t row = start + t0 + lane;
        const float bb = __bfloat162float(p.b[row * p.ld_ba + h]);
        const float aa = __bfloat162float(p.a[row * p.ld_ba + h]);
        bs[lane] = 1.f / (1.f + __expf(-bb));
        gs[lane] = __expf(a_log * softplus(aa + dtb));  // decay exp(g), g = -exp(A_log) softplus(a + dt_bias)
      }
#pragma unroll
      for (int t = 0; t < TCHUNK; ++t) {
        if (t < nt) {
          const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qw[t]);
          const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kw[t]);
          const float2 qa = __bfloat1622float2(q2[0]), qb = __bfloat1622float2(q2[1]);
          const float2 ka = __bfloat1622float2(k2[0]), kb = __bfloat1622float2(k2[1]);
          float sq = qa.x * qa.x + qa.y * qa.y + qb.x * qb.x + qb.y * qb.y;
          float sk = ka.x * ka.x + ka.y * ka.y + kb.x * kb.x + kb.y * kb.y;
          float sqk = qa.x * ka.x + qa.y * ka.y + qb.x * kb.x + qb.y * kb.y;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
            sqk += __shfl_xor_sync(0xffffffffu, sqk, o);
          }
          const float nq = rsqrtf(sq + 1e-6f) * p.q_scale, nk = rsqrtf(sk + 1e-6f);
          *reinterpret_cast<float4*>(&qs[t][kidx(lane * 4)]) = make_float4(qa.x * nq, qa.y * nq, qb.x * nq, qb.y * nq);
          *reinterpret_cast<float4*>(&ks[t][kidx(lane * 4)]) = make_float4(ka.x * nk, ka.y * nk, kb.x * nk, kb.y * nk);
          if (lane == 0) qk[t] = sqk * nq * nk;
          if (!half) vs[t][jj] = vr[t];
        }
      }
      __syncwarp();
#pragma unroll 1
      for (int t = 0; t < nt; ++t) {
        const int row = start + t0 + t;
        const float vj = vs[t][jj];
        const float dec = gs[t];
        float k0 = 0.f, k1 = 0.f, k2 = 0.f, k3 = 0.f, q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
#pragma unroll
        for (int i = 0; i < HALF; i += 4) {
          const float4 kk = *reinterpret_cast<const float4*>(&ks[t][kidx(r0 + i)]);
          const float4 qq = *reinterpret_cast<const float4*>(&qs[t][kidx(r0 + i)]);
          k0 = fmaf(S[i], kk.x, k0);
          k1 = fmaf(S[i + 1], kk.y, k1);
          k2 = fmaf(S[i + 2], kk.z, k2);
          k3 = fmaf(S[i + 3], kk.w, k3);
          q0 = fmaf(S[i], qq.x, q0);
          q1 = fmaf(S[i + 1], qq.y, q1);
          q2 = fmaf(S[i + 2], qq.z, q2);
          q3 = fmaf(S[i + 3], qq.w, q3);
        }
        float kS = (k0 + k1) + (k2 + k3), qS = (q0 + q1) + (q2 + q3);
        kS += __shfl_xor_sync(0xffffffffu, kS, 1);
        qS += __shfl_xor_sync(0xffffffffu, qS, 1);
        const float u = bs[t] * (vj - dec * kS);
        if (!half) p.out[static_cast<int64_t>(row) * p.ld_out + h * DK + col] = __float2bfloat16_rn(dec * qS + qk[t] * u);
#pragma unroll
        for (int i = 0; i < HALF; i += 4) {
          const float4 kk = *reinterpret_cast<const float4*>(&ks[t][kidx(r0 + i)]);
          S[i] = fmaf(dec, S[i], kk.x * u);
          S[i + 1] = fmaf(dec, S[i + 1], kk.y * u);
          S[i + 2] = fmaf(dec, S[i + 2], kk.z * u);
          S[i + 3] = fmaf(dec, S[i + 3], kk.w * u);
        }
      }
    }
    if (ri == 0 && sg.save_slot >= 0) {  // state after the cached prefix -> the pool slot
      float* st = p.state_pool + static_cast<int64_t>(sg.save_slot) * p.slot_stride +
                  static_cast<int64_t>(h) * DK * DK + static_cast<int64_t>(r0) * DK + col;
#pragma unroll
      for (int i = 0; i < HALF; ++i) st[static_cast<int64_t>(i) * DK] = S[i];
    }
    if (ri == 1 && sg.n_branches > 1) {
#pragma unroll
      for (int i = 0; i < HALF; ++i) fork[r0 + i][jj] = S[i];
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
  dim3 grid(dv / delta::COLS, hv, n_segs);
  delta::gated_delta_scan_kernel<<<grid, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
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
