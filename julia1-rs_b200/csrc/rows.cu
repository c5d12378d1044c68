// Row kernels that do not fold into a GEMM epilogue: embedding gather + LayerNorm,
// the encoder final norm + question-type embedding + first head norm, row gathers
// for marker rows, and the one-time FP32 -> BF16 weight conversion.
// One warp per row; H is a template parameter (H / 128 float4 per lane).
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace j1rt {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int H>
struct Row {
  static constexpr int V = H / 128;  // float4 per lane
  float4 v[V];

  __device__ __forceinline__ void load(const float* __restrict__ p, int lane) {
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = *reinterpret_cast<const float4*>(p + j * 128 + lane * 4);
  }
  __device__ __forceinline__ void store(float* __restrict__ p, int lane) const {
#pragma unroll
    for (int j = 0; j < V; ++j) *reinterpret_cast<float4*>(p + j * 128 + lane * 4) = v[j];
  }
  __device__ __forceinline__ void store_bf16(bf16* __restrict__ p, int lane) const {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      uint2 q;
      q.x = pack_bf16x2(v[j].x, v[j].y);
      q.y = pack_bf16x2(v[j].z, v[j].w);
      *reinterpret_cast<uint2*>(p + j * 128 + lane * 4) = q;
    }
  }
  __device__ __forceinline__ void add(const float* __restrict__ p, int lane) {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float4 q = *reinterpret_cast<const float4*>(p + j * 128 + lane * 4);
      v[j].x += q.x;
      v[j].y += q.y;
      v[j].z += q.z;
      v[j].w += q.w;
    }
  }
  // Two-pass LayerNorm (mean, then mean squared deviation), as kernels.cu:19-41.
  __device__ __forceinline__ void layer_norm(const float* __restrict__ w, const float* __restrict__ b, float eps,
                                             int lane) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) s += v[j].x + v[j].y + v[j].z + v[j].w;
    const float mean = warp_sum(s) * (1.f / H);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float a = v[j].x - mean, c = v[j].y - mean, d = v[j].z - mean, e = v[j].w - mean;
      q += a * a + c * c + d * d + e * e;
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.f / H) + eps);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int i = j * 128 + lane * 4;
      const float4 g = *reinterpret_cast<const float4*>(w + i);
      const float4 bb = b ? *reinterpret_cast<const float4*>(b + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[j].x = (v[j].x - mean) * rstd * g.x + bb.x;
      v[j].y = (v[j].y - mean) * rstd * g.y + bb.y;
      v[j].z = (v[j].z - mean) * rstd * g.z + bb.z;
      v[j].w = (v[j].w - mean) * rstd * g.w + bb.w;
    }
  }
};

// x = LayerNorm(table[id]) (no bias); xn = bf16(x): layer 0 has no attention norm.
template <int H>
__global__ void __launch_bounds__(256) embed_ln_kernel(const int* __restrict__ ids, const float* __restrict__ table,
                                                       const float* __restrict__ w, float* __restrict__ x,
                                                       bf16* __restrict__ xn, int rows, float eps) {
  grid_dep_launch();
  grid_dep_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  Row<H> r;
  r.load(table + static_cast<size_t>(ids[row]) * H, lane);
  r.layer_norm(w, nullptr, eps, lane);
  r.store(x + static_cast<size_t>(row) * H, lane);
  r.store_bf16(xn + static_cast<size_t>(row) * H, lane);
}

// x = LN_final(x) (no bias) + type_emb[qtype]; xn = bf16(LN(x; hw, hb, 1e-5)).
template <int H>
__global__ void __launch_bounds__(256) final_norm_kernel(float* __restrict__ x, const float* __restrict__ fw,
                                                         const float* __restrict__ type_emb,
                                                         const int* __restrict__ qtype, const float* __restrict__ hw,
                                                         const float* __restrict__ hb, bf16* __restrict__ xn,
                                                         int rows, float eps) {
  grid_dep_launch();
  grid_dep_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  Row<H> r;
  float* xr = x + static_cast<size_t>(row) * H;
  r.load(xr, lane);
  r.layer_norm(fw, nullptr, eps, lane);
  r.add(type_emb + static_cast<size_t>(qtype[row]) * H, lane);
  r.store(xr, lane);
  r.layer_norm(hw, hb, 1e-5f, lane);
  r.store_bf16(xn + static_cast<size_t>(row) * H, lane);
}

__global__ void __launch_bounds__(256) gather_rows_kernel(const uint8_t* __restrict__ src, const int* __restrict__ idx,
                                                          uint8_t* __restrict__ dst, int rows, int row_bytes) {
  grid_dep_launch();
  grid_dep_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<size_t>(idx[row]) * row_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + static_cast<size_t>(row) * row_bytes);
  for (int i = lane; i < row_bytes / 16; i += 32) d[i] = s[i];
}

// dst row r <- src row perm(r); with geglu_inter = I > 0 the [2I, K] Wi is
// re-laid out so 256-row tile t holds gate-input rows 128t.. and gate rows I+128t..
__global__ void f32_to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, long long rows, int cols,
                                   int geglu_inter) {
  const long long n = rows * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols, c = i % cols;
    long long sr = r;
    if (geglu_inter > 0) {
      const long long t = r / 256, h = (r % 256) / 128, k = r % 128;
      sr = h * geglu_inter + t * 128 + k;
    }
    dst[i] = __float2bfloat16_rn(src[sr * cols + c]);
  }
}

template <int H>
int embed_ln_h(const int* ids, const float* table, const float* w, float* x, bf16* xn, int rows, float eps,
               cudaStream_t st) {
  return static_cast<int>(launch_kernel(embed_ln_kernel<H>, dim3((rows + 7) / 8), dim3(256), 0, st, ids, table, w, x,
                                        xn, rows, eps));
}
template <int H>
int final_norm_h(float* x, const float* fw, const float* te, const int* qt, const float* hw, const float* hb,
                 bf16* xn, int rows, float eps, cudaStream_t st) {
  return static_cast<int>(launch_kernel(final_norm_kernel<H>, dim3((rows + 7) / 8), dim3(256), 0, st, x, fw, te, qt,
                                        hw, hb, xn, rows, eps));
}

}  // namespace

bool hidden_supported(int hidden) { return hidden == 256 || hidden == 384 || hidden == 512 || hidden == 768 || hidden == 1024; }

int launch_embed_ln(int hidden, const int* ids, const float* table, const float* w, float* x, bf16* xn, int rows,
                    float eps, cudaStream_t st) {
  if (rows == 0) return 0;
  switch (hidden) {
    case 256: return embed_ln_h<256>(ids, table, w, x, xn, rows, eps, st);
    case 384: return embed_ln_h<384>(ids, table, w, x, xn, rows, eps, st);
    case 512: return embed_ln_h<512>(ids, table, w, x, xn, rows, eps, st);
    case 768: return embed_ln_h<768>(ids, table, w, x, xn, rows, eps, st);
    case 1024: return embed_ln_h<1024>(ids, table, w, x, xn, rows, eps, st);
  }
  return static_cast<int>(cudaErrorInvalidValue);
}

int launch_final_norm(int hidden, float* x, const float* fw, const float* te, const int* qt, const float* hw,
                      const float* hb, bf16* xn, int rows, float eps, cudaStream_t st) {
  if (rows == 0) return 0;
  switch (hidden) {
    case 256: return final_norm_h<256>(x, fw, te, qt, hw, hb, xn, rows, eps, st);
    case 384: return final_norm_h<384>(x, fw, te, qt, hw, hb, xn, rows, eps, st);
    case 512: return final_norm_h<512>(x, fw, te, qt, hw, hb, xn, rows, eps, st);
    case 768: return final_norm_h<768>(x, fw, te, qt, hw, hb, xn, rows, eps, st);
    case 1024: return final_norm_h<1024>(x, fw, te, qt, hw, hb, xn, rows, eps, st);
  }
  return static_cast<int>(cudaErrorInvalidValue);
}

int launch_gather_rows(const void* src, const int* idx, void* dst, int rows, int row_bytes, cudaStream_t st) {
  if (rows == 0) return 0;
  return static_cast<int>(launch_kernel(gather_rows_kernel, dim3((rows + 7) / 8), dim3(256), 0, st,
                                        static_cast<const uint8_t*>(src), idx, static_cast<uint8_t*>(dst), rows,
                                        row_bytes));
}

int launch_f32_to_bf16(const float* src, bf16* dst, long long rows, int cols, int geglu_inter, cudaStream_t st) {
  if (rows == 0 || cols == 0) return 0;
  const long long n = rows * cols;
  long long blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  f32_to_bf16_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(src, dst, rows, cols, geglu_inter);
  return static_cast<int>(cudaGetLastError());
}

namespace {
__global__ void wait_timeout_selftest_kernel(int* err, long long limit) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_for(&bar, 0, &abort_flag, err, 99, limit);  // nothing ever arrives
}
}  // namespace

int launch_wait_timeout_selftest(int* err, long long limit, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(err, limit);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace j1rt
