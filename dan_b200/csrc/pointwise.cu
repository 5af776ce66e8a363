// Stand-alone forms of element-wise steps that the model path fuses into other kernels:
// SwiGLU (fused into the gate/up GEMM's epilogue there), the Gated DeltaNet gates (fused into
// the scan), the exact log-sum-exp merge of two partial attention results (which the single
// tree-attention kernel never needs), and e4m3 quantisation with one scale for the whole tensor
// (dan's path for GPUs whose row-wise scaled matmul is slow). They back the Python functions
// that keep dan's fused.py names and signatures, so code written against those functions runs
// on B200 unchanged. All are HBM-bound one-pass kernels over bf16 rows with the reference's
// rounding points.
#include "common.cuh"

namespace dan {
namespace pw {

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// y = bf16(bf16(silu(g)) * u): F.silu(gate) * up in bf16 (dan/fused.py:59-61), one rounding
// after the activation and one after the product.
__global__ void swiglu_kernel(const __nv_bfloat16* g, int64_t ldg, const __nv_bfloat16* u, int64_t ldu,
                              __nv_bfloat16* y, int64_t ldy, int rows, int cols) {
  const int64_t n = static_cast<int64_t>(rows) * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const float gv = __bfloat162float(g[r * ldg + c]);
    const float uv = __bfloat162float(u[r * ldu + c]);
    y[r * ldy + c] = __float2bfloat16_rn(bf16r(gv / (1.f + expf(-gv))) * uv);
  }
}

// beta = bf16(sigmoid(b)); g = -exp(A_log) * softplus(a + dt_bias) in fp32, softplus linear
// above 20 as torch's (dan/fused.py:79-82).
__global__ void delta_gates_kernel(const __nv_bfloat16* b, int64_t ldb, const __nv_bfloat16* a, int64_t lda,
                                   const float* a_log, const float* dt_bias, __nv_bfloat16* beta, int64_t ldbeta,
                                   float* g, int64_t ldg, int rows, int heads) {
  const int64_t n = static_cast<int64_t>(rows) * heads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / heads;
    const int h = static_cast<int>(i % heads);
    const float bv = __bfloat162float(b[r * ldb + h]);
    beta[r * ldbeta + h] = __float2bfloat16_rn(1.f / (1.f + expf(-bv)));
    const float x = __bfloat162float(a[r * lda + h]) + dt_bias[h];
    const float sp = x > 20.f ? x : log1pf(expf(x));
    g[r * ldg + h] = -expf(a_log[h]) * sp;
  }
}

// out = bf16((o_a e^{la - m} + o_b e^{lb - m}) / (e^{la - m} + e^{lb - m})), m = max(la, lb),
// o [T, H, D] bf16 (row stride ldo, head stride D), lse [H, T] fp32 (dan/fused.py:94-101).
__global__ void lse_merge_kernel(const __nv_bfloat16* oa, const float* la, const __nv_bfloat16* ob, const float* lb,
                                 __nv_bfloat16* out, int64_t ldo, int t_rows, int heads, int d) {
  const int64_t n = static_cast<int64_t>(t_rows) * heads * d;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / (static_cast<int64_t>(heads) * d);
    const int h = static_cast<int>((i / d) % heads), c = static_cast<int>(i % d);
    const float xa = la[static_cast<int64_t>(h) * t_rows + t], xb = lb[static_cast<int64_t>(h) * t_rows + t];
    const float m = fmaxf(xa, xb);
    const float wa = expf(xa - m), wb = expf(xb - m);
    const int64_t o = t * ldo + static_cast<int64_t>(h) * d + c;
    out[o] = __float2bfloat16_rn((__bfloat162float(oa[o]) * wa + __bfloat162float(ob[o]) * wb) / (wa + wb));
  }
}

// |x| maximum of the whole tensor into *amax (non-negative floats order like their bit
// patterns, so an integer atomicMax suffices; *amax starts at 0).
__global__ void amax_kernel(const __nv_bfloat16* x, int64_t ldx, int rows, int cols, float* amax) {
  const int64_t n = static_cast<int64_t>(rows) * cols;
  float m = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[(i / cols) * ldx + i % cols])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(m));
}

// q = e4m3(x / s), s = max(amax, 1e-12) / 448 (dan/fused.py:85-91 with rowwise=False).
__global__ void quant_tensor_kernel(const __nv_bfloat16* x, int64_t ldx, uint8_t* q, int64_t ldq, int rows, int cols,
                                    const float* amax) {
  const float s = fmaxf(*amax, 1e-12f) / 448.f;
  const float r = __frcp_rn(s);
  const int64_t n = static_cast<int64_t>(rows) * cols / 2;  // pairs (cols is even)
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = 2 * i, row = e / cols, c = e % cols;
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(x + row * ldx + c);
    const float2 f = __bfloat1622float2(v);
    *reinterpret_cast<uint16_t*>(q + row * ldq + c) = static_cast<uint16_t>(e4m3x2_div(f.x, f.y, s, r));
  }
}

__global__ void amax_to_scale_kernel(float* v) { *v = fmaxf(*v, 1e-12f) / 448.f; }

unsigned grid_for(int64_t n) {
  const int64_t blocks = (n + 255) / 256;
  return static_cast<unsigned>(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

}  // namespace pw
}  // namespace dan

using namespace dan;

DAN_API int dan_swiglu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out, int64_t ldo, int rows,
                       int cols, void* stream) {
  DAN_REQUIRE(rows >= 0 && cols > 0 && ldg >= cols && ldu >= cols && ldo >= cols, "swiglu: bad shape or strides");
  if (!rows) return 0;
  pw::swiglu_kernel<<<pw::grid_for(static_cast<int64_t>(rows) * cols), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gate), ldg, static_cast<const __nv_bfloat16*>(up), ldu,
      static_cast<__nv_bfloat16*>(out), ldo, rows, cols);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_delta_gates(const void* b, int64_t ldb, const void* a, int64_t lda, const float* a_log,
                            const float* dt_bias, void* beta, int64_t ldbeta, float* g, int64_t ldg, int rows,
                            int heads, void* stream) {
  DAN_REQUIRE(rows >= 0 && heads > 0 && ldb >= heads && lda >= heads && ldbeta >= heads && ldg >= heads,
              "delta_gates: bad shape or strides");
  if (!rows) return 0;
  pw::delta_gates_kernel<<<pw::grid_for(static_cast<int64_t>(rows) * heads), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(b), ldb, static_cast<const __nv_bfloat16*>(a), lda, a_log, dt_bias,
      static_cast<__nv_bfloat16*>(beta), ldbeta, g, ldg, rows, heads);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_lse_merge(const void* o_a, const float* lse_a, const void* o_b, const float* lse_b, void* out,
                          int64_t ld_row, int t_rows, int heads, int head_dim, void* stream) {
  DAN_REQUIRE(t_rows >= 0 && heads > 0 && head_dim > 0 && ld_row >= static_cast<int64_t>(heads) * head_dim,
              "lse_merge: bad shape or strides");
  if (!t_rows) return 0;
  pw::lse_merge_kernel<<<pw::grid_for(static_cast<int64_t>(t_rows) * heads * head_dim), 256, 0,
                         static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(o_a), lse_a, static_cast<const __nv_bfloat16*>(o_b), lse_b,
      static_cast<__nv_bfloat16*>(out), ld_row, t_rows, heads, head_dim);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API int dan_quantize_e4m3_tensor(const void* x, int64_t ldx, void* q, int64_t ldq, float* scale, int rows,
                                     int cols, void* stream) {
  DAN_REQUIRE(rows >= 0 && cols > 0 && cols % 2 == 0 && ldx % 2 == 0 && ldq % 2 == 0 && ldx >= cols && ldq >= cols,
              "quantize_e4m3_tensor: cols and strides must be even");
  DAN_REQUIRE((reinterpret_cast<uintptr_t>(x) & 3) == 0 && (reinterpret_cast<uintptr_t>(q) & 1) == 0,
              "quantize_e4m3_tensor: x must be 4-byte and q 2-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DAN_CUDA(cudaMemsetAsync(scale, 0, sizeof(float), st));
  const int64_t n = static_cast<int64_t>(rows) * cols;
  if (n) {
    pw::amax_kernel<<<pw::grid_for(n), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx, rows, cols, scale);
    pw::quant_tensor_kernel<<<pw::grid_for(n / 2), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                                  static_cast<uint8_t*>(q), ldq, rows, cols, scale);
  }
  pw::amax_to_scale_kernel<<<1, 1, 0, st>>>(scale);
  DAN_CUDA(cudaGetLastError());
  return 0;
}
