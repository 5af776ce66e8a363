// Memory-bound kernels of the read path: embedding gather, RMSNorm (Llama and
// zero-centred, optionally fused with per-row e4m3 quantisation), RoPE, per-row
// e4m3 quantisation, sigmoid output gate, prefix K/V page stores, and the fused
// final-norm + label gather-GEMV + per-question softmax readout.
//
// All use 128-bit vector loads where rows allow it, one warp per row for the
// row reductions, and compute in fp32 with the reference's rounding points.
#include "common.cuh"

namespace dan {
namespace ew {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------- embedding
__global__ void embed_kernel(const int64_t* ids, const __nv_bfloat16* table, int64_t ldt, int64_t vocab,
                             __nv_bfloat16* out, int64_t ldo, int rows, int cols, int32_t* status) {
  const int row = blockIdx.x;
  int64_t id = ids[row];
  if (id < 0 || id >= vocab) {
    report(status, kBadIndex);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * ldt);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * ldo);
  for (int i = threadIdx.x; i < cols / 8; i += blockDim.x) dst[i] = src[i];
}

// ---------------------------------------------------------------- RMSNorm
// Rows are addressed as (outer, inner): element (r, c) of the logical [rows, cols]
// matrix is at base + (r / inner) * ld_outer + (r % inner) * ld_inner + c, so
// per-head norms run in place on a packed q/k/v buffer.
// mode 0 (Llama, fused.py:35-40):  y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))
// mode 1 (zero-centred, fused.py:43-48): y = bf16(x * rsqrt(mean(x^2) + eps) * (1 + w))
// With ``q8`` set, y is also quantised per row to e4m3 (fused.py:85-91):
//   scale = max(amax |y|, 1e-12) / 448, q = e4m3(y / scale).
// Wide rows (hidden-size norms): 128 threads per row, two rows per block, VPT 16-byte vectors
// per thread, the sum of squares (and the e4m3 amax) reduced through shared memory. Small
// per-thread state keeps many rows in flight per SM, so loads, arithmetic and stores of
// different blocks overlap. Mode 0 writes w * bf16(x * inv) with one rounded bf16 product per
// pair (the exact product of two bf16 values fits in fp32, so this equals the fp32 product
// rounded to bf16); mode 1 bf16(x * inv * (1 + w)) in fp32.
template <int VPT, bool Q8>
__global__ void __launch_bounds__(256) rms_norm_wide_kernel(const __nv_bfloat16* x, int64_t x_outer, int64_t x_inner,
                                                             int inner, const __nv_bfloat16* w, float eps, int mode,
                                                             __nv_bfloat16* y, int64_t y_outer, int64_t y_inner,
                                                             uint8_t* q8, int64_t ldq, float* q8_scale, int rows,
                                                             int cols) {
  __shared__ float red[2][4];
  const int rg = threadIdx.x >> 7, t = threadIdx.x & 127, wg = t >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 2 + rg;
  const bool live = r < rows;
  const int rr = live ? r : 0;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(rr / inner) * x_outer + static_cast<int64_t>(rr % inner) * x_inner;
  __nv_bfloat16* yr = y ? y + static_cast<int64_t>(rr / inner) * y_outer + static_cast<int64_t>(rr % inner) * y_inner
                        : nullptr;
  const int nvec = cols / 8;
  uint4 buf[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = t + 128 * i;
    if (live && v < nvec) {
      buf[i] = reinterpret_cast<const uint4*>(xr)[v];
      const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&buf[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(e[k]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[rg][wg] = ss;
  __syncthreads();
  const float inv = rsqrtf((red[rg][0] + red[rg][1] + red[rg][2] + red[rg][3]) / cols + eps);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = t + 128 * i;
    if (live && v < nvec) {
      __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(&buf[i]);
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + v);
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(e[k]);
        if (mode == 0) {
          e[k] = __hmul2(__floats2bfloat162_rn(f.x * inv, f.y * inv), w2[k]);
        } else {
          const float2 wf = __bfloat1622float2(w2[k]);
          e[k] = __floats2bfloat162_rn(f.x * inv * (1.f + wf.x), f.y * inv * (1.f + wf.y));
        }
        if (Q8) {
          const float2 o = __bfloat1622float2(e[k]);
          amax = fmaxf(amax, fmaxf(fabsf(o.x), fabsf(o.y)));
        }
      }
      if (yr) reinterpret_cast<uint4*>(yr)[v] = buf[i];
    }
  }
  if (Q8) {
    amax = warp_max(amax);
    __syncthreads();  // every thread has read the sum of squares
    if (lane == 0) red[rg][wg] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(red[rg][0], red[rg][1]), fmaxf(red[rg][2], red[rg][3]));
    const float scale = fmaxf(amax, 1e-12f) / 448.f, rcp = __frcp_rn(scale);
    if (live) {
      uint8_t* qr = q8 + static_cast<int64_t>(r) * ldq;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int v = t + 128 * i;
        if (v < nvec) reinterpret_cast<uint2*>(qr)[v] = e4m3x8_div(buf[i], scale, rcp);
      }
      if (t == 0) q8_scale[r] = scale;
    }
  }
}

// MAXV: 16-byte vectors per lane (a row holds at most 32 * MAXV * 8 elements); Q8: also
// quantise the normalised row to e4m3 (the per-row amax is tracked only then).
template <int MAXV, bool Q8>
__global__ void rms_norm_kernel(const __nv_bfloat16* x, int64_t x_outer, int64_t x_inner, int inner,
                                const __nv_bfloat16* w, float eps, int mode, __nv_bfloat16* y, int64_t y_outer,
                                int64_t y_inner, uint8_t* q8, int64_t ldq, float* q8_scale, int rows, int cols) {
  const int warps = blockDim.x / 32;
  const int r = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(r / inner) * x_outer + static_cast<int64_t>(r % inner) * x_inner;
  __nv_bfloat16* yr = y + static_cast<int64_t>(r / inner) * y_outer + static_cast<int64_t>(r % inner) * y_inner;
  const int nvec = cols / 8;
  uint4 buf[MAXV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      buf[i] = reinterpret_cast<const uint4*>(xr)[v];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&buf[i]);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float f = __bfloat162float(e[t]);
        ss += f * f;
      }
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / cols + eps);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&buf[i]);
      const uint4 wv = reinterpret_cast<const uint4*>(w)[v];
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float f = __bfloat162float(e[t]) * inv;
        float o;
        if (mode == 0)
          o = __bfloat162float(we[t]) * bf16_round(f);
        else
          o = f * (1.f + __bfloat162float(we[t]));
        e[t] = __float2bfloat16_rn(o);
        if (Q8) amax = fmaxf(amax, fabsf(__bfloat162float(e[t])));
      }
      if (y) reinterpret_cast<uint4*>(yr)[v] = buf[i];
    }
  }
  if (Q8) {
    amax = warp_max(amax);
    const float scale = fmaxf(amax, 1e-12f) / 448.f, rcp = __frcp_rn(scale);
    uint8_t* qr = q8 + static_cast<int64_t>(r) * ldq;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int v = lane + 32 * i;
      if (v < nvec) reinterpret_cast<uint2*>(qr)[v] = e4m3x8_div(buf[i], scale, rcp);
    }
    if (lane == 0) q8_scale[r] = scale;
  }
}

// ---------------------------------------------------------------- per-row e4m3
// scale = max(amax |x|, 1e-12) / 448 ; q = e4m3(x / scale)   (fused.py:85-91, quant.py:26-33)
// Rows of up to TPR * VPT 16-byte vectors: TPR threads per row (128 or 256), 256 / TPR rows
// per block; each thread issues its VPT loads of the row at once and keeps the row in
// registers, so the row is read once and the amax, then the codes, come from registers.
template <int VPT, int TPR>
__global__ void __launch_bounds__(256) quant_rows_vec_kernel(const __nv_bfloat16* x, int64_t ldx, uint8_t* q,
                                                             int64_t ldq, float* scale, int rows, int cols) {
  constexpr int W = TPR / 32;  // warps per row
  __shared__ float red[256 / TPR][W];
  const int rg = threadIdx.x / TPR, t = threadIdx.x % TPR, wg = t >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * (256 / TPR) + rg;
  const bool live = r < rows;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(live ? r : 0) * ldx;
  const int nvec = cols / 8;
  uint4 buf[VPT];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = t + TPR * i;
    if (live && v < nvec) buf[i] = reinterpret_cast<const uint4*>(xr)[v];
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = t + TPR * i;
    if (live && v < nvec) {
      const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&buf[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(e[k]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  amax = warp_max(amax);
  if (lane == 0) red[rg][wg] = amax;
  __syncthreads();
  amax = red[rg][0];
#pragma unroll
  for (int k = 1; k < W; ++k) amax = fmaxf(amax, red[rg][k]);
  if (!live) return;
  const float s = fmaxf(amax, 1e-12f) / 448.f, rcp = __frcp_rn(s);
  uint8_t* qr = q + static_cast<int64_t>(r) * ldq;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = t + TPR * i;
    if (v < nvec) reinterpret_cast<uint2*>(qr)[v] = e4m3x8_div(buf[i], s, rcp);
  }
  if (t == 0) scale[r] = s;
}

// Rows longer than 16384 columns: one block per row, the row read twice (amax, then codes).
__global__ void quant_rows_kernel(const __nv_bfloat16* x, int64_t ldx, uint8_t* q, int64_t ldq, float* scale,
                                  int rows, int cols) {
  const int r = blockIdx.x;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(r) * ldx;
  __shared__ float red[32];
  float amax = 0.f;
  for (int c = threadIdx.x * 8; c < cols; c += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int t = 0; t < 8; ++t) amax = fmaxf(amax, fabsf(__bfloat162float(e[t])));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float a = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    a = warp_max(a);
    if (threadIdx.x == 0) red[0] = fmaxf(a, 1e-12f) / 448.f;
  }
  __syncthreads();
  const float s = red[0], rcp = __frcp_rn(s);
  if (threadIdx.x == 0) scale[r] = s;
  uint8_t* qr = q + static_cast<int64_t>(r) * ldq;
  for (int c = threadIdx.x * 8; c < cols; c += blockDim.x * 8)
    *reinterpret_cast<uint2*>(qr + c) = e4m3x8_div(*reinterpret_cast<const uint4*>(xr + c), s, rcp);
}

// ---------------------------------------------------------------- RoPE
// cos/sin table, once per forward: angle = float(pos) * inv_freq[i] in fp32, then cos and
// sin rounded to bf16 as the reference does (llama.py:155-158, qwen3_5.py:411-414).
__global__ void rope_table_kernel(const int64_t* pos, const float* inv_freq, int rows, int half, float* cos_t,
                                  float* sin_t) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * half) return;
  const int r = static_cast<int>(idx / half), i = static_cast<int>(idx % half);
  const float ang = static_cast<float>(pos[r]) * inv_freq[i];
  float sn, cs;
  sincosf(ang, &sn, &cs);
  cos_t[idx] = bf16_round(cs);
  sin_t[idx] = bf16_round(sn);
}

// Rotate-half on the first ``rot`` dims of each head, in place, 8 pairs per thread with
// 16-byte accesses (llama.py:43-45, fused.py:69-76); products and sum rounded to bf16 at
// the reference's points.
__global__ void rope_kernel(__nv_bfloat16* x, int64_t ld_row, int64_t ld_head, int heads, int rot,
                            const float* cos_t, const float* sin_t, int rows) {
  const int half = rot / 2, groups = half / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * heads * groups) return;
  const int r = static_cast<int>(idx / (heads * groups));
  const int rem = static_cast<int>(idx % (heads * groups));
  const int h = rem / groups, i0 = (rem % groups) * 8;
  __nv_bfloat16* p = x + static_cast<int64_t>(r) * ld_row + static_cast<int64_t>(h) * ld_head;
  uint4 va = *reinterpret_cast<const uint4*>(p + i0), vb = *reinterpret_cast<const uint4*>(p + half + i0);
  __nv_bfloat16* ea = reinterpret_cast<__nv_bfloat16*>(&va);
  __nv_bfloat16* eb = reinterpret_cast<__nv_bfloat16*>(&vb);
  const float* ct = cos_t + static_cast<int64_t>(r) * half + i0;
  const float* st = sin_t + static_cast<int64_t>(r) * half + i0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const float a = __bfloat162float(ea[t]), b = __bfloat162float(eb[t]);
    const float c = ct[t], s = st[t];
    ea[t] = __float2bfloat16_rn(bf16_round(a * c) + bf16_round(-b * s));
    eb[t] = __float2bfloat16_rn(bf16_round(b * c) + bf16_round(a * s));
  }
  *reinterpret_cast<uint4*>(p + i0) = va;
  *reinterpret_cast<uint4*>(p + half + i0) = vb;
}

// ---------------------------------------------------------------- sigmoid gate
// o[r, j] = bf16(o[r, j] * sigmoid(g[r, j]))  (fused.py:64-66); g row stride may differ.
__global__ void sigmoid_gate_kernel(__nv_bfloat16* o, int64_t ldo, const __nv_bfloat16* g, int64_t ldg,
                                    int64_t g_head_stride, int head_dim, int rows, int cols) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * cols) return;
  const int r = static_cast<int>(idx / cols), c = static_cast<int>(idx % cols);
  const float gv = __bfloat162float(g[static_cast<int64_t>(r) * ldg + (c / head_dim) * g_head_stride + c % head_dim]);
  const float ov = __bfloat162float(o[static_cast<int64_t>(r) * ldo + c]);
  o[static_cast<int64_t>(r) * ldo + c] = __float2bfloat16_rn(ov * (1.f / (1.f + __expf(-gv))));
}

// Vector form: one thread per 8 consecutive columns of a head (16-byte loads and store); used
// when rows, heads and strides are 16-byte aligned.
__global__ void sigmoid_gate_vec_kernel(__nv_bfloat16* o, int64_t ldo, const __nv_bfloat16* g, int64_t ldg,
                                        int64_t g_head_stride, int head_dim, int rows, int cols) {
  const int vcols = cols / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * vcols) return;
  const int r = static_cast<int>(idx / vcols), c = static_cast<int>(idx % vcols) * 8;
  uint4* op = reinterpret_cast<uint4*>(o + static_cast<int64_t>(r) * ldo + c);
  const uint4 gv = *reinterpret_cast<const uint4*>(g + static_cast<int64_t>(r) * ldg + (c / head_dim) * g_head_stride +
                                                   c % head_dim);
  uint4 ov = *op;
  const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 gf = __bfloat1622float2(g2[i]), of = __bfloat1622float2(o2[i]);
    o2[i] = __floats2bfloat162_rn(of.x * (1.f / (1.f + __expf(-gf.x))), of.y * (1.f / (1.f + __expf(-gf.y))));
  }
  *op = ov;
}

// ---------------------------------------------------------------- prefix K/V page store
// Copies rows src_rows[i] of k/v ([rows, heads, d] strided) to pool rows dst_rows[i].
__global__ void kv_store_kernel(const __nv_bfloat16* k, const __nv_bfloat16* v, int64_t ld_row, int64_t ld_head,
                                __nv_bfloat16* pk, __nv_bfloat16* pv, int64_t pld_row, int64_t pld_head,
                                const int* src_rows, const int* dst_rows, int count, int heads, int d) {
  const int i = blockIdx.x;
  if (i >= count) return;
  const int64_t s = src_rows[i], t = dst_rows[i];
  const int vec = d / 8;
  for (int e = threadIdx.x; e < heads * vec; e += blockDim.x) {
    const int h = e / vec, c = (e % vec) * 8;
    *reinterpret_cast<uint4*>(pk + t * pld_row + h * pld_head + c) =
        *reinterpret_cast<const uint4*>(k + s * ld_row + h * ld_head + c);
    *reinterpret_cast<uint4*>(pv + t * pld_row + h * pld_head + c) =
        *reinterpret_cast<const uint4*>(v + s * ld_row + h * ld_head + c);
  }
}

// ---------------------------------------------------------------- label readout
// One thread-block cluster of C CTAs per question (C = 1..8, from the launch's largest label
// count): every CTA norms the question's read row (the norm is row-wise, so norming only the
// read rows equals norming all rows then gathering, llama.py:161 + runner.py:73), computes the
// logits W_lm[label] . h in fp32 (llama.py:163-165) of its contiguous share of the labels (one
// label row per warp at a time, the whole 8 KB row's loads in flight), and the question's
// softmax (readout.py:13-17) is combined across the cluster through distributed shared memory:
// each CTA publishes its (max, sum of exp) and reads its peers'. One CTA per question had left
// most SMs idle (24-48 questions per batch) and each warp's label rows in flight one 2 KB slice
// at a time (0.28 / 0.65 TB/s of label bytes on configuration-3 / -5 label counts under ncu).
constexpr int kReadoutThreads = 512;

__device__ __forceinline__ float dot_row(const __nv_bfloat16* wr, const float* sh, int hidden, int lane) {
  float acc = 0.f;
  // 16 x 16 bytes per lane in flight per round: a 4096-wide row in one round.
  for (int c0 = lane * 8; c0 < hidden; c0 += 16 * 256) {
    uint4 v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (c0 + 256 * u < hidden) v[u] = __ldcs(reinterpret_cast<const uint4*>(wr + c0 + 256 * u));
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int c = c0 + 256 * u;
      if (c >= hidden) break;
      const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(e[t]);
        acc = fmaf(f.x, sh[c + 2 * t], acc);
        acc = fmaf(f.y, sh[c + 2 * t + 1], acc);
      }
    }
  }
  return warp_sum(acc);
}

__global__ void __launch_bounds__(kReadoutThreads) readout_kernel(
    const __nv_bfloat16* h, int64_t ldh, const int* read_rows, const __nv_bfloat16* nw, float eps, int mode,
    const __nv_bfloat16* wlm, int64_t ldw, int64_t vocab, const int* label_ids, const int* offsets, int hidden,
    int max_labels, float* logits, float* probs, int32_t* status) {
  extern __shared__ float sh[];  // [hidden] normed row, then this CTA's share of the logits
  __shared__ float red[32];
  __shared__ float stat[2];  // this CTA's (max, sum of exp(logit - max)) for its peers
  const int q = blockIdx.y;
  const int crank = static_cast<int>(cluster_rank()), csize = static_cast<int>(gridDim.x);
  const int nwarps = blockDim.x / 32, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* x = h + static_cast<int64_t>(read_rows[q]) * ldh;
  float ss = 0.f;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    const float f = __bfloat162float(x[c]);
    sh[c] = f;
    ss += f * f;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nwarps ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = rsqrtf(t / hidden + eps);
  }
  __syncthreads();
  const float inv = red[0];
  if (mode != 2) {  // mode 2: the row is already final-normed (label_logits on a hidden state)
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float f = sh[c] * inv;
      const float w = __bfloat162float(nw[c]);
      sh[c] = bf16_round(mode == 0 ? w * bf16_round(f) : f * (1.f + w));
    }
  }
  __syncthreads();
  const int a = offsets[q];
  int b = offsets[q + 1];
  if (b < a || b - a > max_labels) {  // the output slots hold max_labels values: clamp, report
    if (threadIdx.x == 0 && crank == 0) report(status, kBadIndex);
    b = b < a ? a : a + max_labels;
  }
  const int per = (b - a + csize - 1) / csize;
  const int lo = min(b, a + crank * per), hi = min(b, lo + per);
  float* lg = sh + hidden;
  for (int j = lo + warp; j < hi; j += nwarps) {
    int64_t id = label_ids[j];
    if (id < 0 || id >= vocab) {
      report(status, kBadIndex);
      id = 0;
    }
    const float acc = dot_row(wlm + id * ldw, sh, hidden, lane);
    if (lane == 0) lg[j - lo] = acc;
  }
  __syncthreads();
  if (warp == 0) {
    float mx = -INFINITY;
    for (int j = lane; j < hi - lo; j += 32) mx = fmaxf(mx, lg[j]);
    mx = warp_max(mx);
    float z = 0.f;
    for (int j = lane; j < hi - lo; j += 32) z += expf(lg[j] - mx);
    z = warp_sum(z);
    if (lane == 0) {
      stat[0] = mx;
      stat[1] = z;
    }
  }
  cluster_sync();  // every CTA's (max, sum) is published
  if (warp == 0) {
    float m = -INFINITY, z = 0.f;
    if (lane < csize) {
      const uint32_t base = map_shared(smem_u32(stat), static_cast<uint32_t>(lane));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(m) : "r"(base));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(z) : "r"(base + 4));
    }
    const float big = warp_max(m);
    float part = (z > 0.f) ? z * expf(m - big) : 0.f;
    part = warp_sum(part);
    for (int j = lane; j < hi - lo; j += 32) {
      logits[lo + j] = lg[j];
      probs[lo + j] = expf(lg[j] - big) / part;
    }
  }
  cluster_sync();  // peers keep their shared memory until every CTA has read it
}

}  // namespace ew
}  // namespace dan

using namespace dan;

DAN_API int dan_embed(const int64_t* ids, const void* table, int64_t ldt, int64_t vocab, void* out, int64_t ldo,
                      int rows, int cols, int32_t* status, void* stream) {
  DAN_REQUIRE(rows >= 0 && cols > 0 && cols % 8 == 0 && ldt % 8 == 0 && ldo % 8 == 0,
              "embed: cols/ld must be multiples of 8");
  if (!rows) return 0;
  ew::embed_kernel<<<rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      ids, static_cast<const __nv_bfloat16*>(table), ldt, vocab, static_cast<__nv_bfloat16*>(out), ldo, rows, cols,
      status);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_rms_norm(const void* x, int64_t x_outer, int64_t x_inner, int inner, const void* w, float eps,
                         int mode, void* y, int64_t y_outer, int64_t y_inner, void* q8, int64_t ldq, float* q8_scale,
                         int rows, int cols, void* stream) {
  DAN_REQUIRE(cols > 0 && cols % 8 == 0 && cols <= 8192, "rms_norm: cols=%d must be a multiple of 8 <= 8192", cols);
  DAN_REQUIRE(inner > 0 && (mode == 0 || mode == 1), "rms_norm: bad inner=%d or mode=%d", inner, mode);
  DAN_REQUIRE(x_outer % 8 == 0 && x_inner % 8 == 0 && y_outer % 8 == 0 && y_inner % 8 == 0,
              "rms_norm: strides must be multiples of 8");
  DAN_REQUIRE(y || q8, "rms_norm: no output");
  if (!rows) return 0;
  cudaStream_t s0 = static_cast<cudaStream_t>(stream);
  if (cols >= 2048) {  // hidden-size rows: 128 threads per row
    const int vpt = (cols / 8 + 127) / 128;
    const dim3 g2((rows + 1) / 2);
    const auto* xw = static_cast<const __nv_bfloat16*>(x);
    const auto* ww = static_cast<const __nv_bfloat16*>(w);
    auto* yw = static_cast<__nv_bfloat16*>(y);
    auto* qw = static_cast<uint8_t*>(q8);
#define DAN_WIDE(V)                                                                                                 \
  do {                                                                                                              \
    if (qw)                                                                                                         \
      ew::rms_norm_wide_kernel<V, true><<<g2, 256, 0, s0>>>(xw, x_outer, x_inner, inner, ww, eps, mode, yw, y_outer, \
                                                            y_inner, qw, ldq, q8_scale, rows, cols);                  \
    else                                                                                                            \
      ew::rms_norm_wide_kernel<V, false><<<g2, 256, 0, s0>>>(xw, x_outer, x_inner, inner, ww, eps, mode, yw,       \
                                                             y_outer, y_inner, qw, ldq, q8_scale, rows, cols);      \
  } while (0)
    if (vpt <= 2)
      DAN_WIDE(2);
    else if (vpt <= 4)
      DAN_WIDE(4);
    else
      DAN_WIDE(8);
#undef DAN_WIDE
    DAN_CUDA(cudaGetLastError());
    return 0;
  }
  const int warps = 8;
  const int per_lane = (cols / 8 + 31) / 32;
  const dim3 grid((rows + warps - 1) / warps), block(32 * warps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* yb = static_cast<__nv_bfloat16*>(y);
  auto* qb = static_cast<uint8_t*>(q8);
#define DAN_NORM(NV)                                                                                            \
  do {                                                                                                          \
    if (qb)                                                                                                     \
      ew::rms_norm_kernel<NV, true><<<grid, block, 0, s>>>(xb, x_outer, x_inner, inner, wb, eps, mode, yb, y_outer, \
                                                           y_inner, qb, ldq, q8_scale, rows, cols);             \
    else                                                                                                        \
      ew::rms_norm_kernel<NV, false><<<grid, block, 0, s>>>(xb, x_outer, x_inner, inner, wb, eps, mode, yb,        \
                                                            y_outer, y_inner, qb, ldq, q8_scale, rows, cols);   \
  } while (0)
  if (per_lane <= 1)
    DAN_NORM(1);
  else if (per_lane <= 2)
    DAN_NORM(2);
  else if (per_lane <= 4)
    DAN_NORM(4);
  else if (per_lane <= 8)
    DAN_NORM(8);
  else if (per_lane <= 16)
    DAN_NORM(16);
  else
    DAN_NORM(32);
#undef DAN_NORM
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_quantize_e4m3(const void* x, int64_t ldx, void* q, int64_t ldq, float* scale, int rows, int cols,
                              void* stream) {
  DAN_REQUIRE(cols > 0 && cols % 8 == 0 && ldx % 8 == 0 && ldq % 16 == 0, "quantize_e4m3: bad cols/ld");
  DAN_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 7) == 0,
              "quantize_e4m3: x must be 16-byte and q 8-byte aligned");
  if (!rows) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* qb = static_cast<uint8_t*>(q);
  // Measured at M = 3400 (graph-timed): 14336 columns 28.8 us, 4096 columns 8.5 us (two-pass
  // block-per-row kernel 37.3 / 10.5 us; HBM time 22 / 6.3 us).
  const int nvec = cols / 8;
  const dim3 g2((rows + 1) / 2);
  if (nvec <= 128 * 2)
    ew::quant_rows_vec_kernel<2, 128><<<g2, 256, 0, st>>>(xb, ldx, qb, ldq, scale, rows, cols);
  else if (nvec <= 128 * 4)
    ew::quant_rows_vec_kernel<4, 128><<<g2, 256, 0, st>>>(xb, ldx, qb, ldq, scale, rows, cols);
  else if (nvec <= 128 * 8)
    ew::quant_rows_vec_kernel<8, 128><<<g2, 256, 0, st>>>(xb, ldx, qb, ldq, scale, rows, cols);
  else if (nvec <= 256 * 8)
    ew::quant_rows_vec_kernel<8, 256><<<rows, 256, 0, st>>>(xb, ldx, qb, ldq, scale, rows, cols);
  else
    ew::quant_rows_kernel<<<rows, 256, 0, st>>>(xb, ldx, qb, ldq, scale, rows, cols);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_rope_table(const int64_t* pos, const float* inv_freq, int rows, int half, float* cos_t,
                           float* sin_t, void* stream) {
  DAN_REQUIRE(half > 0, "rope_table: half=%d", half);
  if (!rows) return 0;
  const int64_t n = static_cast<int64_t>(rows) * half;
  ew::rope_table_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      pos, inv_freq, rows, half, cos_t, sin_t);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_rope(void* x, int64_t ld_row, int64_t ld_head, int heads, int head_dim, int rot, const float* cos_t,
                     const float* sin_t, int rows, void* stream) {
  DAN_REQUIRE(rot > 0 && rot % 16 == 0 && rot <= head_dim, "rope: rot=%d must be a multiple of 16 <= head_dim=%d",
              rot, head_dim);
  DAN_REQUIRE(ld_row % 8 == 0 && ld_head % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0,
              "rope: x must be 16-byte aligned with strides that are multiples of 8");
  if (!rows || !heads) return 0;
  const int64_t n = static_cast<int64_t>(rows) * heads * (rot / 16);
  ew::rope_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(x), ld_row, ld_head, heads, rot, cos_t, sin_t, rows);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_sigmoid_gate(void* o, int64_t ldo, const void* g, int64_t ldg, int64_t g_head_stride, int head_dim,
                             int rows, int cols, void* stream) {
  if (!rows) return 0;
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (a16(o) && a16(g) && cols % 8 == 0 && head_dim % 8 == 0 && ldo % 8 == 0 && ldg % 8 == 0 &&
      g_head_stride % 8 == 0) {
    const int64_t nv = static_cast<int64_t>(rows) * (cols / 8);
    ew::sigmoid_gate_vec_kernel<<<static_cast<unsigned>((nv + 255) / 256), 256, 0,
                                  static_cast<cudaStream_t>(stream)>>>(
        static_cast<__nv_bfloat16*>(o), ldo, static_cast<const __nv_bfloat16*>(g), ldg, g_head_stride, head_dim, rows,
        cols);
    DAN_CUDA(cudaGetLastError());
    return 0;
  }
  const int64_t n = static_cast<int64_t>(rows) * cols;
  ew::sigmoid_gate_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(o), ldo, static_cast<const __nv_bfloat16*>(g), ldg, g_head_stride, head_dim, rows,
      cols);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_kv_store(const void* k, const void* v, int64_t ld_row, int64_t ld_head, void* pool_k, void* pool_v,
                         int64_t pool_row, int64_t pool_head, const int* src_rows, const int* dst_rows, int count,
                         int heads, int head_dim, void* stream) {
  DAN_REQUIRE(head_dim % 8 == 0 && ld_row % 8 == 0 && ld_head % 8 == 0 && pool_row % 8 == 0 && pool_head % 8 == 0,
              "kv_store: strides must be multiples of 8");
  if (!count) return 0;
  ew::kv_store_kernel<<<count, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), ld_row, ld_head,
      static_cast<__nv_bfloat16*>(pool_k), static_cast<__nv_bfloat16*>(pool_v), pool_row, pool_head, src_rows,
      dst_rows, count, heads, head_dim);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_label_readout(const void* h, int64_t ldh, const int* read_rows, const void* norm_w, float eps,
                              int mode, const void* w_lm, int64_t ldw, int64_t vocab, const int* label_ids,
                              const int* offsets, int n_questions, int hidden, int max_labels, float* logits,
                              float* probs, int32_t* status, void* stream) {
  DAN_REQUIRE(hidden > 0 && hidden % 8 == 0 && ldw % 8 == 0, "label_readout: hidden/ldw must be multiples of 8");
  DAN_REQUIRE(max_labels >= 0 && max_labels <= 4096, "label_readout: at most 4096 labels per question");
  DAN_REQUIRE(mode >= 0 && mode <= 2, "label_readout: unknown norm mode %d", mode);
  DAN_REQUIRE(n_questions >= 0 && n_questions < 65536, "label_readout: %d questions", n_questions);
  if (!n_questions) return 0;
  // Cluster size: about 16 labels per CTA (one per warp), at most the portable 8.
  int csize = (max_labels + 15) / 16;
  csize = csize < 1 ? 1 : (csize > 8 ? 8 : csize);
  const int per = (max_labels + csize - 1) / csize;
  const size_t smem = (static_cast<size_t>(hidden) + (per > 0 ? per : 1)) * sizeof(float);
  DAN_REQUIRE(smem <= 200 * 1024, "label_readout: hidden %d too large", hidden);
  static std::atomic<uint64_t> configured{0};
  if (smem > 48 * 1024) DAN_CUDA(smem_limit_once(ew::readout_kernel, 200 * 1024, configured));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(csize), static_cast<unsigned>(n_questions), 1);
  cfg.blockDim = dim3(ew::kReadoutThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DAN_CUDA(cudaLaunchKernelEx(&cfg, ew::readout_kernel, static_cast<const __nv_bfloat16*>(h), ldh, read_rows,
                              static_cast<const __nv_bfloat16*>(norm_w), eps, mode,
                              static_cast<const __nv_bfloat16*>(w_lm), ldw, vocab, label_ids, offsets, hidden,
                              max_labels, logits, probs, status));
  return 0;
}
