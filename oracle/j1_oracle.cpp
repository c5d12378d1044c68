// TEST INFRASTRUCTURE ONLY -- the parity oracle and timed CPU baseline.
// Never linked into or called by the product (libj1); only tests/, the smoke
// check and bench.py's CPU-baseline leg load this library.
//
// Two CPU restatements of the reference julia1-rs forward over a packed batch:
//
//  mode 0  FP32 "CPU path": src/cpu/mod.rs:201-340 (forward_packed) with
//          src/cpu/gemm.rs (32-column packed panels, 8x32 register tile held over
//          all of K, fused Store/Add/Bias/BiasRelu/AddBias and GEGLU epilogues)
//          and src/cpu/fastmath.rs (Cephes-style exp, rational erf, exact-erf GELU).
//          RoPE in place after the QKV product, softmax_range with the fast exp,
//          two-pass LayerNorm with 16-lane partial sums, last head layer on
//          marker queries only.
//
//  mode 1  BF16 "CUDA path": src/cuda/mod.rs:446-511 with src/cuda/kernels.cu.
//          GEMM operands and outputs rounded to BF16 at exactly the reference's
//          points (xn, qkv, ctx, delta, h, g, RoPE'd q/k, P), FP32 accumulation,
//          FP32 residual stream, residual adds inside the next LayerNorm, and the
//          attention kernel's 64-query tiles / 64-key blocks online softmax in
//          base 2 (kernels.cu:272-381).
//
// Parity pins for this file: the reference's own unit-test protocols
// (src/cpu/gemm.rs:377-426 naive-f64 GEMM/GEGLU at 1e-4; src/cpu/fastmath.rs:51-77
// exp/erf error bounds) are restated in tests/test_oracle.py, and mode 1 is checked
// on the GPU against the reference's own kernels.cu compiled unmodified (hidden 384).
#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

// ---------------------------------------------------------------- fastmath (src/cpu/fastmath.rs)
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

inline float fast_exp(float x) {  // fastmath.rs:8-23
  x = std::min(std::max(x, -87.3f), 88.3f);
  volatile float shifted_v = x * 1.44269504088896340736f + kRoundMagic;  // keep the rounding trick un-fused
  const float shifted = shifted_v;
  const float n = shifted - kRoundMagic;
  const float r = x - n * 0.6933594f - n * -2.1219444e-4f;
  float y = 1.9875691e-4f;
  y = y * r + 1.3982e-3f;
  y = y * r + 8.333452e-3f;
  y = y * r + 4.1665796e-2f;
  y = y * r + 1.6666665e-1f;
  y = y * r + 5e-1f;
  y = y * r * r + r + 1.0f;
  uint32_t sb, mb;
  std::memcpy(&sb, &shifted, 4);
  const float magic = kRoundMagic;
  std::memcpy(&mb, &magic, 4);
  const uint32_t n_int = sb - mb;
  const uint32_t scale_bits = (n_int + 127u) << 23;
  float scale;
  std::memcpy(&scale, &scale_bits, 4);
  return y * scale;
}

inline float fast_erf(float x) {  // fastmath.rs:27-43 (Eigen/XLA float rational approximation)
  x = std::min(std::max(x, -4.0f), 4.0f);
  const float x2 = x * x;
  float p = -2.7261423e-10f;
  p = p * x2 + 2.7706814e-8f;
  p = p * x2 + -2.101024e-6f;
  p = p * x2 + -5.6925064e-5f;
  p = p * x2 + -7.3499063e-4f;
  p = p * x2 + -2.9546e-3f;
  p = p * x2 + -1.6096033e-2f;
  float q = -1.4566072e-5f;
  q = q * x2 + -2.1337406e-4f;
  q = q * x2 + -1.682827e-3f;
  q = q * x2 + -7.373329e-3f;
  q = q * x2 + -1.426474e-2f;
  return x * p / q;
}

inline float fast_gelu(float x) { return 0.5f * x * (1.0f + fast_erf(x * 0.70710678118654752440f)); }
// kernels.cu:134 (libm erff on the device path)
inline float erf_gelu(float x) { return 0.5f * x * (1.f + std::erf(x * 0.70710678118654752f)); }

inline float bf16r(float v) {  // round to nearest even, as half::bf16::from_f32 / __float2bfloat16_rn
  uint32_t b;
  std::memcpy(&b, &v, 4);
  if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x7FFFFFu)) return v;  // NaN
  b += 0x7FFFu + ((b >> 16) & 1u);
  b &= 0xFFFF0000u;
  float r;
  std::memcpy(&r, &b, 4);
  return r;
}

// ---------------------------------------------------------------- reductions (src/cpu/mod.rs:593-617)
inline float sum16(const float* x, size_t n) {
  float acc[16] = {0};
  size_t i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; ++j) acc[j] += x[i + j];
  float s = 0.f;
  for (int j = 0; j < 16; ++j) s += acc[j];
  float r = 0.f;
  for (; i < n; ++i) r += x[i];
  return s + r;
}
inline float max16(const float* x, size_t n) {
  float acc[16];
  for (int j = 0; j < 16; ++j) acc[j] = -INFINITY;
  size_t i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; ++j) acc[j] = std::max(acc[j], x[i + j]);
  float m = -INFINITY;
  for (int j = 0; j < 16; ++j) m = std::max(m, acc[j]);
  for (; i < n; ++i) m = std::max(m, x[i]);
  return m;
}

// layer_norm (src/cpu/mod.rs:620-646)
void layer_norm_cpu(const float* x, const float* w, const float* b, float eps, float* out, size_t n) {
  const float nf = static_cast<float>(n);
  const float mean = sum16(x, n) / nf;
  float acc[16] = {0};
  size_t i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; ++j) {
      const float d = x[i + j] - mean;
      acc[j] += d * d;
    }
  float s = 0.f;
  for (int j = 0; j < 16; ++j) s += acc[j];
  float r = 0.f;
  for (; i < n; ++i) r += (x[i] - mean) * (x[i] - mean);
  const float var = (s + r) / nf;
  const float rstd = 1.0f / std::sqrt(var + eps);
  for (size_t k = 0; k < n; ++k) out[k] = b ? (x[k] - mean) * rstd * w[k] + b[k] : (x[k] - mean) * rstd * w[k];
}

void rows_layer_norm(const float* x, const float* w, const float* b, float eps, float* out, size_t rows, size_t h) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(rows); ++r) layer_norm_cpu(x + r * h, w, b, eps, out + r * h, h);
}

// ln_row of kernels.cu:19-41 (mean then mean squared deviation, rsqrt) on one row.
void layer_norm_gpu(const float* x, const float* w, const float* b, float eps, float* out, size_t n) {
  float s = 0.f;
  for (size_t k = 0; k < n; ++k) s += x[k];
  const float mean = s * (1.f / static_cast<float>(n));
  float q = 0.f;
  for (size_t k = 0; k < n; ++k) q += (x[k] - mean) * (x[k] - mean);
  const float rstd = 1.f / std::sqrt(q * (1.f / static_cast<float>(n)) + eps);
  for (size_t k = 0; k < n; ++k) out[k] = (x[k] - mean) * rstd * w[k] + (b ? b[k] : 0.f);
}

// ---------------------------------------------------------------- GEMM (src/cpu/gemm.rs)
constexpr int NR = 32, MR = 8;

bool have_avx512() {
  static const bool v = __builtin_cpu_supports("avx512f");
  return v;
}

// A [n, k] row-major weight packed into 32-column panels [k][32] (zero padded past n).
struct PackedW {
  std::vector<float> panels;
  size_t n = 0, k = 0;
  void pack(const float* w, size_t n_, size_t k_, bool round_bf16) {
    n = n_, k = k_;
    const size_t np = (n + NR - 1) / NR;
    panels.assign(np * k * NR, 0.f);
#pragma omp parallel for schedule(static)
    for (long long p = 0; p < static_cast<long long>(np); ++p)
      for (size_t kk = 0; kk < k; ++kk)
        for (int j = 0; j < NR; ++j) {
          const size_t col = p * NR + j;
          if (col < n) {
            const float v = w[col * k + kk];
            panels[(p * k + kk) * NR + j] = round_bf16 ? bf16r(v) : v;
          }
        }
  }
  const float* panel(size_t p) const { return panels.data() + p * k * NR; }
};

__attribute__((target("avx512f"))) void tile_avx512(size_t k, const float* a, size_t lda, const float* b,
                                                     float* tile) {
  __m512 acc[MR][2];
  for (int i = 0; i < MR; ++i) acc[i][0] = acc[i][1] = _mm512_setzero_ps();
  for (size_t kk = 0; kk < k; ++kk) {
    const __m512 b0 = _mm512_loadu_ps(b + kk * NR), b1 = _mm512_loadu_ps(b + kk * NR + 16);
    for (int i = 0; i < MR; ++i) {
      const __m512 av = _mm512_set1_ps(a[i * lda + kk]);
      acc[i][0] = _mm512_fmadd_ps(av, b0, acc[i][0]);
      acc[i][1] = _mm512_fmadd_ps(av, b1, acc[i][1]);
    }
  }
  for (int i = 0; i < MR; ++i) {
    _mm512_storeu_ps(tile + i * NR, acc[i][0]);
    _mm512_storeu_ps(tile + i * NR + 16, acc[i][1]);
  }
}

void tile_scalar(size_t k, const float* a, size_t lda, const float* b, float* tile) {
  for (int i = 0; i < MR * NR; ++i) tile[i] = 0.f;
  for (size_t kk = 0; kk < k; ++kk)
    for (int i = 0; i < MR; ++i) {
      const float av = a[i * lda + kk];
      for (int j = 0; j < NR; ++j) tile[i * NR + j] = std::fma(av, b[kk * NR + j], tile[i * NR + j]);
    }
}

inline void tile8x32(size_t k, const float* a, size_t lda, const float* b, float* tile) {
  if (have_avx512()) tile_avx512(k, a, lda, b, tile);
  else tile_scalar(k, a, lda, b, tile);
}

enum Epi { STORE = 0, ADD = 1, BIAS = 2, BIAS_RELU = 3, ADD_BIAS = 4 };

// Product of MR rows starting at r (zero-padded copy for a short strip).
inline void strip_product(const float* x, size_t rows, size_t k, size_t r, const float* panel, float* tile,
                          std::vector<float>& pad) {
  const size_t mr = std::min<size_t>(MR, rows - r);
  if (mr == MR) {
    tile8x32(k, x + r * k, k, panel, tile);
  } else {
    pad.assign(MR * k, 0.f);
    std::memcpy(pad.data(), x + r * k, mr * k * 4);
    tile8x32(k, pad.data(), k, panel, tile);
  }
}

// out[r, col .. col+n] = epi(x[r, :k] . W^T)   (gemm.rs:171-206)
void linear(const float* x, size_t rows, const PackedW& w, float* out, size_t ldo, size_t col, Epi epi,
            const float* bias) {
  if (rows == 0) return;
  const size_t np = (w.n + NR - 1) / NR;
  const size_t nstrips = (rows + MR - 1) / MR;
#pragma omp parallel
  {
    std::vector<float> pad;
    alignas(64) float tile[MR * NR];
#pragma omp for schedule(dynamic, 4) collapse(2)
    for (long long s = 0; s < static_cast<long long>(nstrips); ++s)
      for (long long p = 0; p < static_cast<long long>(np); ++p) {
        const size_t r = s * MR;
        strip_product(x, rows, w.k, r, w.panel(p), tile, pad);
        const size_t mr = std::min<size_t>(MR, rows - r);
        const size_t ncols = std::min<size_t>(NR, w.n - p * NR);
        for (size_t i = 0; i < mr; ++i) {
          float* dst = out + (r + i) * ldo + col + p * NR;
          const float* t = tile + i * NR;
          for (size_t j = 0; j < ncols; ++j) {
            const float b = bias ? bias[p * NR + j] : 0.f;
            switch (epi) {
              case STORE: dst[j] = t[j]; break;
              case ADD: dst[j] += t[j]; break;
              case BIAS: dst[j] = t[j] + b; break;
              case BIAS_RELU: dst[j] = std::max(t[j] + b, 0.f); break;
              case ADD_BIAS: dst[j] += t[j] + b; break;
            }
          }
        }
      }
  }
}

// g[r, :] = gelu(x.Wa^T) * (x.Wb^T) for a [2*inter, k] weight (gemm.rs:210-249)
void linear_geglu(const float* x, size_t rows, const PackedW& w, float* g) {
  const size_t inter = w.n / 2, half = inter / NR;
  const size_t nstrips = (rows + MR - 1) / MR;
#pragma omp parallel
  {
    std::vector<float> pad;
    alignas(64) float ta[MR * NR], tb[MR * NR];
#pragma omp for schedule(dynamic, 4) collapse(2)
    for (long long s = 0; s < static_cast<long long>(nstrips); ++s)
      for (long long p = 0; p < static_cast<long long>(half); ++p) {
        const size_t r = s * MR;
        strip_product(x, rows, w.k, r, w.panel(p), ta, pad);
        strip_product(x, rows, w.k, r, w.panel(half + p), tb, pad);
        const size_t mr = std::min<size_t>(MR, rows - r);
        for (size_t i = 0; i < mr; ++i)
          for (int j = 0; j < NR; ++j) g[(r + i) * inter + p * NR + j] = fast_gelu(ta[i * NR + j]) * tb[i * NR + j];
      }
  }
}

// ---------------------------------------------------------------- model
struct Config {
  int hidden, heads, intermediate, layers, half_window, vocab, max_positions, head_layers;
  float norm_eps;
};

struct Layer {
  const float *attn_norm, *wqkv, *wo, *mlp_norm, *wi, *wo2;
  PackedW p_qkv, p_wo, p_wi, p_wo2;        // fp32
  PackedW b_qkv, b_wo, b_wi, b_wo2;        // bf16-rounded
  float theta;
  bool global;
};
struct Head {
  const float *n1w, *n1b, *in_w, *in_b, *out_w, *out_b, *n2w, *n2b, *l1w, *l1b, *l2w, *l2b;
  PackedW p_in, p_q, p_kv, p_out, p_l1, p_l2;
  PackedW b_in, b_out, b_l1, b_l2;
};

struct Model {
  Config c;
  const float *emb, *emb_norm, *final_norm, *type_emb;
  std::vector<Layer> layers;
  std::vector<Head> head;
  const float *s_nw, *s_nb, *s_w1, *s_b1, *s_w2;
  float s_b2;
  PackedW p_s1, b_s1;
  std::vector<std::vector<float>> rope_cos, rope_sin;  // per layer (shared content per theta)
  bool packed_fp32 = false, packed_bf16 = false;
};

void rope_table(float theta, int hd, int positions, std::vector<float>& c, std::vector<float>& s) {
  // src/config.rs:99-112
  const int half = hd / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(hd));
  c.assign(static_cast<size_t>(positions) * half, 0.f);
  s.assign(static_cast<size_t>(positions) * half, 0.f);
  for (int p = 0; p < positions; ++p)
    for (int i = 0; i < half; ++i) {
      const float f = inv[i] * static_cast<float>(p);
      c[static_cast<size_t>(p) * half + i] = std::cos(f);
      s[static_cast<size_t>(p) * half + i] = std::sin(f);
    }
}

void ensure_packed(Model* m, bool bf16) {
  const size_t H = m->c.hidden, I = m->c.intermediate, FF = 4 * H;
  if (!bf16 && !m->packed_fp32) {
    for (auto& l : m->layers) {
      l.p_qkv.pack(l.wqkv, 3 * H, H, false);
      l.p_wo.pack(l.wo, H, H, false);
      l.p_wi.pack(l.wi, 2 * I, H, false);
      l.p_wo2.pack(l.wo2, H, I, false);
    }
    for (auto& h : m->head) {
      h.p_in.pack(h.in_w, 3 * H, H, false);
      h.p_q.pack(h.in_w, H, H, false);
      h.p_kv.pack(h.in_w + H * H, 2 * H, H, false);
      h.p_out.pack(h.out_w, H, H, false);
      h.p_l1.pack(h.l1w, FF, H, false);
      h.p_l2.pack(h.l2w, H, FF, false);
    }
    m->p_s1.pack(m->s_w1, H, H, false);
    m->packed_fp32 = true;
  }
  if (bf16 && !m->packed_bf16) {
    for (auto& l : m->layers) {
      l.b_qkv.pack(l.wqkv, 3 * H, H, true);
      l.b_wo.pack(l.wo, H, H, true);
      l.b_wi.pack(l.wi, 2 * I, H, true);
      l.b_wo2.pack(l.wo2, H, I, true);
    }
    for (auto& h : m->head) {
      h.b_in.pack(h.in_w, 3 * H, H, true);
      h.b_out.pack(h.out_w, H, H, true);
      h.b_l1.pack(h.l1w, FF, H, true);
      h.b_l2.pack(h.l2w, H, FF, true);
    }
    m->b_s1.pack(m->s_w1, H, H, true);
    m->packed_bf16 = true;
  }
}

struct Batch {
  const uint32_t* ids;
  size_t t;
  const uint32_t* starts;
  const uint32_t* lens;
  const uint8_t* qtypes;
  size_t nseq;
  const uint32_t* marker_rows;
  const uint32_t* marker_starts;
  size_t m;
};

// Attention over packed sequences (src/cpu/mod.rs:365-429 semantics, FP32):
// for sequence s, query rows q_row[s] .. q_row[s]+nq[s]-1 at positions q_pos0[s]+i
// (positions i when the queries are the sequence itself) attend to key rows
// kv_row[s] .. kv_row[s]+len[s]-1; band |i - j| <= window when window >= 0.
struct ASeq {
  size_t q_row, nq, kv_row, len;
  bool self;  // query i sits at position i
};

void attention_fp32(const float* q, size_t ldq, const float* kv, size_t ldkv, size_t k_off, size_t v_off, float* out,
                    size_t ldo, const std::vector<ASeq>& seqs, int heads, int window, float scale) {
  struct Task {
    size_t s;
    int head;
    size_t q0;
  };
  std::vector<Task> tasks;
  for (size_t s = 0; s < seqs.size(); ++s)
    for (int h = 0; h < heads; ++h)
      for (size_t q0 = 0; q0 < seqs[s].nq; q0 += 64) tasks.push_back({s, h, q0});
#pragma omp parallel
  {
    std::vector<float> sc;
#pragma omp for schedule(dynamic, 1)
    for (long long ti = 0; ti < static_cast<long long>(tasks.size()); ++ti) {
      const Task& tk = tasks[ti];
      const ASeq& S = seqs[tk.s];
      const size_t q1 = std::min(tk.q0 + 64, S.nq);
      for (size_t i = tk.q0; i < q1; ++i) {
        size_t lo = 0, hi = S.len;
        if (window >= 0 && S.self) {
          lo = i >= static_cast<size_t>(window) ? i - window : 0;
          hi = std::min(S.len, i + window + 1);
        }
        const float* qi = q + (S.q_row + i) * ldq + tk.head * 64;
        sc.assign(hi - lo, 0.f);
        for (size_t j = lo; j < hi; ++j) {
          const float* kj = kv + (S.kv_row + j) * ldkv + k_off + tk.head * 64;
          float d = 0.f;
          for (int e = 0; e < 64; ++e) d += qi[e] * kj[e];
          sc[j - lo] = d;
        }
        // softmax_range (src/cpu/mod.rs:579-591): exp((s - max) * scale), times 1/sum
        const float mx = max16(sc.data(), sc.size());
        for (auto& v : sc) v = fast_exp((v - mx) * scale);
        const float inv = 1.0f / sum16(sc.data(), sc.size());
        for (auto& v : sc) v *= inv;
        float o[64] = {0};
        for (size_t j = lo; j < hi; ++j) {
          const float* vj = kv + (S.kv_row + j) * ldkv + v_off + tk.head * 64;
          const float p = sc[j - lo];
          for (int e = 0; e < 64; ++e) o[e] += p * vj[e];
        }
        std::memcpy(out + (S.q_row + i) * ldo + tk.head * 64, o, 64 * 4);
      }
    }
  }
}

// Attention of the reference CUDA kernel (kernels.cu:215-381), emulated in FP32 with its
// BF16 rounding points: 64-query tiles, 64-key blocks from kbeg, RoPE on load (rounded
// to bf16), base-2 online softmax with P rounded to bf16 for P.V, O / l rounded to bf16.
void attention_bf16(const float* qkv, size_t t, int H, const Batch& b, int heads, const float* cos_t,
                    const float* sin_t, int window, float* out) {
  const size_t ld = 3 * H;
  const float scale_log2 = 0.125f * 1.44269504088896340736f;
  struct Task {
    size_t s;
    int head;
    int q0;
  };
  std::vector<Task> tasks;
  for (size_t s = 0; s < b.nseq; ++s)
    for (int h = 0; h < heads; ++h)
      for (int q0 = 0; q0 < static_cast<int>(b.lens[s]); q0 += 64) tasks.push_back({s, h, q0});
  (void)t;
#pragma omp parallel
  {
    std::vector<float> Q(64 * 64), K(64 * 64), V(64 * 64);
#pragma omp for schedule(dynamic, 1)
    for (long long ti = 0; ti < static_cast<long long>(tasks.size()); ++ti) {
      const Task& tk = tasks[ti];
      const int start = static_cast<int>(b.starts[tk.s]), len = static_cast<int>(b.lens[tk.s]);
      const float* seq = qkv + static_cast<size_t>(start) * ld + tk.head * 64;
      auto load = [&](std::vector<float>& dst, const float* base, int pos0, bool rope) {
        for (int r = 0; r < 64; ++r) {
          const int p = pos0 + r;
          float* d = dst.data() + r * 64;
          if (p >= len) {
            std::fill(d, d + 64, 0.f);
            continue;
          }
          const float* src = base + static_cast<size_t>(p) * ld;
          if (rope && cos_t) {
            for (int i = 0; i < 32; ++i) {
              const float x = src[i], y = src[i + 32];
              const float c = cos_t[static_cast<size_t>(p) * 32 + i], sn = sin_t[static_cast<size_t>(p) * 32 + i];
              d[i] = bf16r(x * c - y * sn);
              d[i + 32] = bf16r(y * c + x * sn);
            }
          } else {
            std::memcpy(d, src, 64 * 4);
          }
        }
      };
      load(Q, seq, tk.q0, true);
      float o[64][64] = {{0}};
      float m[64], l[64];
      for (int r = 0; r < 64; ++r) m[r] = -INFINITY, l[r] = 0.f;
      int kbeg = 0, kend = len;
      if (window >= 0) {
        kbeg = std::max(0, tk.q0 - window);
        kend = std::min(len, tk.q0 + 64 + window);
      }
      for (int k0 = kbeg; k0 < kend; k0 += 64) {
        load(K, seq + H, k0, true);
        load(V, seq + 2 * H, k0, false);
        for (int r = 0; r < 64; ++r) {
          const int row = tk.q0 + r;
          float s[64];
          float mx = -INFINITY;
          for (int c = 0; c < 64; ++c) {
            const int key = k0 + c;
            float d = 0.f;
            for (int e = 0; e < 64; ++e) d += Q[r * 64 + e] * K[c * 64 + e];
            const bool ok = key < kend && (window < 0 || std::abs(row - key) <= window);
            s[c] = ok ? d * scale_log2 : -INFINITY;
            mx = std::max(mx, s[c]);
          }
          const float n = std::max(m[r], mx);
          const float u = n == -INFINITY ? 0.f : n;
          const float a = std::exp2(m[r] - u);
          m[r] = n;
          l[r] *= a;
          for (int e = 0; e < 64; ++e) o[r][e] *= a;
          for (int c = 0; c < 64; ++c) {
            const float p = std::exp2(s[c] - u);
            l[r] += p;
            const float pb = bf16r(p);
            if (pb != 0.f)
              for (int e = 0; e < 64; ++e) o[r][e] += pb * V[c * 64 + e];
          }
        }
      }
      for (int r = 0; r < 64; ++r) {
        const int row = tk.q0 + r;
        if (row >= len) continue;
        const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
        float* dst = out + static_cast<size_t>(start + row) * H + tk.head * 64;
        for (int e = 0; e < 64; ++e) dst[e] = bf16r(o[r][e] * inv);
      }
    }
  }
}

void round_all(float* v, size_t n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < static_cast<long long>(n); ++i) v[i] = bf16r(v[i]);
}

// ---------------------------------------------------------------- FP32 CPU path (mode 0)
void forward_fp32(Model* M, const Batch& b, float* scores, float* hidden_out) {
  ensure_packed(M, false);
  const Config& c = M->c;
  const size_t H = c.hidden, I = c.intermediate, FF = 4 * H, t = b.t, m = b.m;
  std::vector<float> x(t * H), xn(t * H), qkv(t * 3 * H), ctx(t * H), g(t * I), h(t * FF);
  std::vector<uint32_t> pos(t);
  {
    size_t o = 0;
    for (size_t s = 0; s < b.nseq; ++s)
      for (uint32_t p = 0; p < b.lens[s]; ++p) pos[o++] = p;
  }
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(t); ++r)
    layer_norm_cpu(M->emb + static_cast<size_t>(b.ids[r]) * H, M->emb_norm, nullptr, c.norm_eps, &x[r * H], H);
  std::vector<ASeq> seqs;
  for (size_t s = 0; s < b.nseq; ++s) seqs.push_back({b.starts[s], b.lens[s], b.starts[s], b.lens[s], true});
  for (int l = 0; l < c.layers; ++l) {
    Layer& L = M->layers[l];
    const float* normed = x.data();
    if (L.attn_norm) {
      rows_layer_norm(x.data(), L.attn_norm, nullptr, c.norm_eps, xn.data(), t, H);
      normed = xn.data();
    }
    linear(normed, t, L.p_qkv, qkv.data(), 3 * H, 0, STORE, nullptr);
    // rope_inplace (src/cpu/mod.rs:343-360)
    const float* ct = M->rope_cos[l].data();
    const float* st = M->rope_sin[l].data();
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < static_cast<long long>(t); ++r) {
      const float* cc = ct + static_cast<size_t>(pos[r]) * 32;
      const float* ss = st + static_cast<size_t>(pos[r]) * 32;
      float* row = &qkv[r * 3 * H];
      for (size_t hh = 0; hh < 2 * H; hh += 64)
        for (int i = 0; i < 32; ++i) {
          const float a = row[hh + i], bb = row[hh + 32 + i];
          row[hh + i] = a * cc[i] - bb * ss[i];
          row[hh + 32 + i] = bb * cc[i] + a * ss[i];
        }
    }
    attention_fp32(qkv.data(), 3 * H, qkv.data(), 3 * H, H, 2 * H, ctx.data(), H, seqs, c.heads,
                   L.global ? -1 : c.half_window, 0.125f);
    linear(ctx.data(), t, L.p_wo, x.data(), H, 0, ADD, nullptr);
    rows_layer_norm(x.data(), L.mlp_norm, nullptr, c.norm_eps, xn.data(), t, H);
    linear_geglu(xn.data(), t, L.p_wi, g.data());
    linear(g.data(), t, L.p_wo2, x.data(), H, 0, ADD, nullptr);
  }
  // final norm + question-type embedding
  for (size_t s = 0; s < b.nseq; ++s) {
    const float* te = M->type_emb + static_cast<size_t>(b.qtypes[s]) * H;
#pragma omp parallel for schedule(static)
    for (long long r = b.starts[s]; r < static_cast<long long>(b.starts[s] + b.lens[s]); ++r) {
      std::vector<float> tmp(H);
      layer_norm_cpu(&x[r * H], M->final_norm, nullptr, c.norm_eps, tmp.data(), H);
      if (hidden_out) std::memcpy(hidden_out + r * H, tmp.data(), H * 4);
      for (size_t k = 0; k < H; ++k) x[r * H + k] = tmp[k] + te[k];
    }
  }
  const int nh = static_cast<int>(M->head.size());
  for (int j = 0; j + 1 < nh; ++j) {
    Head& hd = M->head[j];
    rows_layer_norm(x.data(), hd.n1w, hd.n1b, 1e-5f, xn.data(), t, H);
    linear(xn.data(), t, hd.p_in, qkv.data(), 3 * H, 0, BIAS, hd.in_b);
    attention_fp32(qkv.data(), 3 * H, qkv.data(), 3 * H, H, 2 * H, ctx.data(), H, seqs, c.heads, -1, 0.125f);
    linear(ctx.data(), t, hd.p_out, x.data(), H, 0, ADD_BIAS, hd.out_b);
    rows_layer_norm(x.data(), hd.n2w, hd.n2b, 1e-5f, xn.data(), t, H);
    linear(xn.data(), t, hd.p_l1, h.data(), FF, 0, BIAS_RELU, hd.l1b);
    linear(h.data(), t, hd.p_l2, x.data(), H, 0, ADD_BIAS, hd.l2b);
  }
  std::vector<float> y(m * H);
  for (size_t k = 0; k < m; ++k) std::memcpy(&y[k * H], &x[static_cast<size_t>(b.marker_rows[k]) * H], H * 4);
  if (nh > 0) {
    Head& hd = M->head[nh - 1];
    rows_layer_norm(x.data(), hd.n1w, hd.n1b, 1e-5f, xn.data(), t, H);
    linear(xn.data(), t, hd.p_kv, qkv.data(), 3 * H, H, BIAS, hd.in_b + H);  // keys/values for every token
    std::vector<float> xm(m * H), qm(m * H), cm(m * H), yn(m * H), hm(m * FF);
    for (size_t k = 0; k < m; ++k) std::memcpy(&xm[k * H], &xn[static_cast<size_t>(b.marker_rows[k]) * H], H * 4);
    linear(xm.data(), m, hd.p_q, qm.data(), H, 0, BIAS, hd.in_b);  // queries for markers only
    std::vector<ASeq> ms;
    for (size_t s = 0; s < b.nseq; ++s)
      ms.push_back({b.marker_starts[s], static_cast<size_t>(b.marker_starts[s + 1] - b.marker_starts[s]), b.starts[s],
                    b.lens[s], false});
    attention_fp32(qm.data(), H, qkv.data(), 3 * H, H, 2 * H, cm.data(), H, ms, c.heads, -1, 0.125f);
    linear(cm.data(), m, hd.p_out, y.data(), H, 0, ADD_BIAS, hd.out_b);
    rows_layer_norm(y.data(), hd.n2w, hd.n2b, 1e-5f, yn.data(), m, H);
    linear(yn.data(), m, hd.p_l1, hm.data(), FF, 0, BIAS_RELU, hd.l1b);
    linear(hm.data(), m, hd.p_l2, y.data(), H, 0, ADD_BIAS, hd.l2b);
  }
  std::vector<float> yn(m * H), z(m * H);
  rows_layer_norm(y.data(), M->s_nw, M->s_nb, 1e-5f, yn.data(), m, H);
  linear(yn.data(), m, M->p_s1, z.data(), H, 0, BIAS, M->s_b1);
  for (size_t k = 0; k < m; ++k) {
    float acc = 0.f;
    for (size_t i = 0; i < H; ++i) acc += fast_gelu(z[k * H + i]) * M->s_w2[i];
    scores[k] = acc + M->s_b2;
  }
}

// ---------------------------------------------------------------- BF16 CUDA path (mode 1)
// ln_bf16 (kernels.cu:97-109): x += delta (+ pending), store, out = bf16(LN(x; w, b)).
void ln_step(float* x, const float* delta, const float* pending, const float* w, const float* b, float* out,
             size_t rows, size_t H, float eps) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(rows); ++r) {
    float* xr = x + r * H;
    if (delta)
      for (size_t k = 0; k < H; ++k) xr[k] += delta[r * H + k];
    if (pending)
      for (size_t k = 0; k < H; ++k) xr[k] += pending[k];
    std::vector<float> tmp(H);
    layer_norm_gpu(xr, w, b, eps, tmp.data(), H);
    for (size_t k = 0; k < H; ++k) out[r * H + k] = bf16r(tmp[k]);
  }
}

void forward_bf16(Model* M, const Batch& b, float* scores) {
  ensure_packed(M, true);
  const Config& c = M->c;
  const size_t H = c.hidden, I = c.intermediate, FF = 4 * H, t = b.t, m = b.m;
  const float eps = c.norm_eps;
  std::vector<float> x(t * H), xn(t * H), qkv(t * 3 * H), ctx(t * H), hbuf(t * std::max(2 * I, FF)), g(t * I),
      delta(t * H), f32s(t * std::max(3 * H, FF));
  // embed_ln (kernels.cu:66-75): x = LN(E[id]); xn = bf16(x)
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(t); ++r) {
    layer_norm_gpu(M->emb + static_cast<size_t>(b.ids[r]) * H, M->emb_norm, nullptr, eps, &x[r * H], H);
    for (size_t k = 0; k < H; ++k) xn[r * H + k] = bf16r(x[r * H + k]);
  }
  const float* dptr = nullptr;
  for (int l = 0; l < c.layers; ++l) {
    Layer& L = M->layers[l];
    if (L.attn_norm) ln_step(x.data(), dptr, nullptr, L.attn_norm, nullptr, xn.data(), t, H, eps);
    linear(xn.data(), t, L.b_qkv, qkv.data(), 3 * H, 0, STORE, nullptr);
    round_all(qkv.data(), t * 3 * H);
    attention_bf16(qkv.data(), t, static_cast<int>(H), b, c.heads, M->rope_cos[l].data(), M->rope_sin[l].data(),
                   L.global ? -1 : c.half_window, ctx.data());
    linear(ctx.data(), t, L.b_wo, delta.data(), H, 0, STORE, nullptr);
    round_all(delta.data(), t * H);
    ln_step(x.data(), delta.data(), nullptr, L.mlp_norm, nullptr, xn.data(), t, H, eps);
    linear(xn.data(), t, L.b_wi, hbuf.data(), 2 * I, 0, STORE, nullptr);
    round_all(hbuf.data(), t * 2 * I);
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < static_cast<long long>(t); ++r)
      for (size_t k = 0; k < I; ++k)
        g[r * I + k] = bf16r(erf_gelu(hbuf[r * 2 * I + k]) * hbuf[r * 2 * I + I + k]);
    linear(g.data(), t, L.b_wo2, delta.data(), H, 0, STORE, nullptr);
    round_all(delta.data(), t * H);
    dptr = delta.data();
  }
  // final_norm (kernels.cu:113-132)
  const Head& h0 = M->head[0];
  std::vector<float> qt(t);
  for (size_t s = 0; s < b.nseq; ++s)
    for (size_t r = b.starts[s]; r < b.starts[s] + b.lens[s]; ++r) qt[r] = b.qtypes[s];
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(t); ++r) {
    float* xr = &x[r * H];
    for (size_t k = 0; k < H; ++k) xr[k] += delta[r * H + k];
    std::vector<float> v(H), o(H);
    layer_norm_gpu(xr, M->final_norm, nullptr, eps, v.data(), H);
    const float* te = M->type_emb + static_cast<size_t>(qt[r]) * H;
    for (size_t k = 0; k < H; ++k) v[k] += te[k], xr[k] = v[k];
    layer_norm_gpu(v.data(), h0.n1w, h0.n1b, 1e-5f, o.data(), H);
    for (size_t k = 0; k < H; ++k) xn[r * H + k] = bf16r(o[k]);
  }
  // decision head (src/cuda/mod.rs:480-507)
  std::vector<float> ym(m * H), ymb(m * H), cm(m * H), dm(m * H), hm(m * FF), zf(m * H);
  const float* pend = nullptr;
  dptr = nullptr;
  float* resid = x.data();
  const int nh = static_cast<int>(M->head.size());
  for (int j = 0; j < nh; ++j) {
    Head& hd = M->head[j];
    if (j > 0) ln_step(x.data(), dptr, pend, hd.n1w, hd.n1b, xn.data(), t, H, 1e-5f);
    linear(xn.data(), t, hd.b_in, f32s.data(), 3 * H, 0, STORE, nullptr);
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < static_cast<long long>(t); ++r)
      for (size_t k = 0; k < 3 * H; ++k) qkv[r * 3 * H + k] = bf16r(f32s[r * 3 * H + k] + hd.in_b[k]);
    attention_bf16(qkv.data(), t, static_cast<int>(H), b, c.heads, nullptr, nullptr, -1, ctx.data());
    if (j + 1 < nh) {
      linear(ctx.data(), t, hd.b_out, delta.data(), H, 0, STORE, nullptr);
      round_all(delta.data(), t * H);
      ln_step(x.data(), delta.data(), hd.out_b, hd.n2w, hd.n2b, xn.data(), t, H, 1e-5f);
      linear(xn.data(), t, hd.b_l1, f32s.data(), FF, 0, STORE, nullptr);
#pragma omp parallel for schedule(static)
      for (long long r = 0; r < static_cast<long long>(t); ++r)
        for (size_t k = 0; k < FF; ++k) hbuf[r * FF + k] = bf16r(std::max(f32s[r * FF + k] + hd.l1b[k], 0.f));
      linear(hbuf.data(), t, hd.b_l2, delta.data(), H, 0, STORE, nullptr);
      round_all(delta.data(), t * H);
      dptr = delta.data();
      pend = hd.l2b;
    } else {
      for (size_t k = 0; k < m; ++k) {
        std::memcpy(&cm[k * H], &ctx[static_cast<size_t>(b.marker_rows[k]) * H], H * 4);
        std::memcpy(&ym[k * H], &x[static_cast<size_t>(b.marker_rows[k]) * H], H * 4);
      }
      linear(cm.data(), m, hd.b_out, dm.data(), H, 0, STORE, nullptr);
      round_all(dm.data(), m * H);
      ln_step(ym.data(), dm.data(), hd.out_b, hd.n2w, hd.n2b, ymb.data(), m, H, 1e-5f);
      linear(ymb.data(), m, hd.b_l1, f32s.data(), FF, 0, STORE, nullptr);
      for (size_t r = 0; r < m; ++r)
        for (size_t k = 0; k < FF; ++k) hm[r * FF + k] = bf16r(std::max(f32s[r * FF + k] + hd.l1b[k], 0.f));
      linear(hm.data(), m, hd.b_l2, dm.data(), H, 0, STORE, nullptr);
      round_all(dm.data(), m * H);
      dptr = dm.data();
      pend = hd.l2b;
      resid = ym.data();
    }
  }
  (void)resid;
  // scorer (src/cuda/mod.rs:508-511; kernels.cu:186-194)
  ln_step(ym.data(), dptr, pend, M->s_nw, M->s_nb, ymb.data(), m, H, 1e-5f);
  linear(ymb.data(), m, M->b_s1, zf.data(), H, 0, STORE, nullptr);
  for (size_t k = 0; k < m; ++k) {
    float s = 0.f;
    for (size_t i = 0; i < H; ++i) s += erf_gelu(zf[k * H + i] + M->s_b1[i]) * M->s_w2[i];
    scores[k] = s + M->s_b2;
  }
}

}  // namespace

// ================================================================== C ABI (test infrastructure)
extern "C" {

typedef struct OracleConfig {
  int hidden, heads, intermediate, layers, half_window, vocab, max_positions, head_layers;
  float norm_eps;
  const int* global;
  const float* rope_theta;
} OracleConfig;

// tensors: in HostWeights::load order (src/model.rs:55-110), see the Python loader.
void* oracle_create(const OracleConfig* cfg, const float* const* tensors, int n_tensors) {
  Model* M = new Model();
  M->c = Config{cfg->hidden, cfg->heads, cfg->intermediate, cfg->layers, cfg->half_window, cfg->vocab,
                cfg->max_positions, cfg->head_layers, cfg->norm_eps};
  int i = 0;
  auto next = [&]() { return i < n_tensors ? tensors[i++] : nullptr; };
  M->emb = next();
  M->emb_norm = next();
  std::vector<std::pair<float, size_t>> tabs;
  for (int l = 0; l < cfg->layers; ++l) {
    Layer L;
    L.attn_norm = l > 0 ? next() : nullptr;
    L.wqkv = next();
    L.wo = next();
    L.mlp_norm = next();
    L.wi = next();
    L.wo2 = next();
    L.theta = cfg->rope_theta[l];
    L.global = cfg->global[l] != 0;
    M->layers.push_back(std::move(L));
  }
  M->final_norm = next();
  M->type_emb = next();
  for (int j = 0; j < cfg->head_layers; ++j) {
    Head h;
    h.n1w = next(), h.n1b = next(), h.in_w = next(), h.in_b = next(), h.out_w = next(), h.out_b = next();
    h.n2w = next(), h.n2b = next(), h.l1w = next(), h.l1b = next(), h.l2w = next(), h.l2b = next();
    M->head.push_back(std::move(h));
  }
  M->s_nw = next(), M->s_nb = next(), M->s_w1 = next(), M->s_b1 = next(), M->s_w2 = next();
  const float* b2 = next();
  if (!b2 || i != n_tensors) {
    delete M;
    return nullptr;
  }
  M->s_b2 = b2[0];
  M->rope_cos.resize(cfg->layers);
  M->rope_sin.resize(cfg->layers);
  for (int l = 0; l < cfg->layers; ++l)
    rope_table(cfg->rope_theta[l], 64, cfg->max_positions, M->rope_cos[l], M->rope_sin[l]);
  return M;
}

void oracle_destroy(void* h) { delete static_cast<Model*>(h); }

// mode 0: FP32 CPU path; mode 1: BF16 CUDA path. hidden_out (mode 0, optional): [t, H]
// LayerNorm_final(x) before the type embedding. threads <= 0: OpenMP default.
int oracle_forward(void* h, int mode, const uint32_t* ids, size_t t, const uint32_t* starts, const uint32_t* lens,
                   const uint8_t* qtypes, size_t nseq, const uint32_t* marker_rows, const uint32_t* marker_starts,
                   size_t m, float* scores, float* hidden_out, int threads) {
  Model* M = static_cast<Model*>(h);
  if (!M) return 1;
  if (threads > 0) omp_set_num_threads(threads);
  Batch b{ids, t, starts, lens, qtypes, nseq, marker_rows, marker_starts, m};
  if (mode == 0) forward_fp32(M, b, scores, hidden_out);
  else forward_bf16(M, b, scores);
  return 0;
}

// gemm.rs `linear` with epilogue 0..4 = Store, Add, Bias, BiasRelu, AddBias (out has row stride ldo, column offset col).
void oracle_linear(const float* x, size_t rows, const float* w, size_t n, size_t k, float* out, size_t ldo, size_t col,
                   int epi, const float* bias, int threads) {
  if (threads > 0) omp_set_num_threads(threads);
  PackedW p;
  p.pack(w, n, k, false);
  linear(x, rows, p, out, ldo, col, static_cast<Epi>(epi), bias);
}

void oracle_linear_geglu(const float* x, size_t rows, const float* w, size_t n2, size_t k, float* g, int threads) {
  if (threads > 0) omp_set_num_threads(threads);
  PackedW p;
  p.pack(w, n2, k, false);
  linear_geglu(x, rows, p, g);
}

float oracle_exp(float x) { return fast_exp(x); }
float oracle_erf(float x) { return fast_erf(x); }
float oracle_gelu(float x) { return fast_gelu(x); }
float oracle_bf16(float x) { return bf16r(x); }
int oracle_has_avx512(void) { return have_avx512() ? 1 : 0; }

}  // extern "C"
