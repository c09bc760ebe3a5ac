// CPU oracle for the pkt MLP training step and the axpy op.
//
// TEST INFRASTRUCTURE ONLY. This library is the checker: it may be loaded by
// tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline / reference
// arm. The product path (pkt_b200) never links, loads or calls it.
//
// What it restates (file:line within Marco-Christiani/pkt):
//   * make_linear_test_data      examples/train_linear.cu:41-76
//   * host_mse                   examples/train_linear.cu:78-86
//   * cpu_train_linear           examples/train_linear.cu:101-151  ("faithful" mode:
//     same loop order, float accumulation, so results are bit-identical to pkt's
//     host loop; pinned against pkt's own binary in tests/golden/)
//   * OpTraits<Axpy>::compute    include/ops/axpy.cuh:33-46 (y = a*x + y; nvcc
//     contracts the expression into one fused multiply-add, so the oracle uses fmaf)
//   * OpTraits<MSELoss>          include/ops/mse.cuh:36-60 (dy = 2(y-t)/(B*m),
//     loss = sum (y-t)^2 / (B*m))
//   * OpTraits<SGDUpdate>        include/ops/sgd.cuh:33-44 (W -= lr*dW)
//   * OpTraits<LinearForward>    include/ops/linear_fwd.cuh:18-29 (y = x W^T)
//   * OpTraits<LinearBackward>   include/ops/linear_bwd.cuh:13-27 (dW = dy^T x, overwrite)
// and extends cpu_train_linear to the multi-layer MLP the B200 engine trains:
// bias, ReLU on hidden layers, dgrad, bias grad, with the operand rounding the
// GPU path applies (bf16 storage / TF32 tensor-core inputs) emulated on the host.
//
// Build: oracle/Makefile (g++ -O3 -fopenmp -shared).

#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

inline float bf16_round(float f) {
  // Round-to-nearest-even to bfloat16, returned as float. NaN kept quiet.
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) {
    u |= 0x00400000u;
    u &= 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
  }
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

inline float tf32_round(float f) {
  // TF32 tensor-core input as the TMA unit produces it from fp32: round to
  // nearest even at 10 mantissa bits (NaN / Inf passed through).
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) {
    u += 0xfffu + ((u >> 13) & 1u);
    u &= 0xffffe000u;
  }
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

enum Mode : int { kFp32 = 0, kTf32 = 1, kBf16 = 2 };

inline float store_round(int mode, float v) { return mode == kBf16 ? bf16_round(v) : v; }
inline float operand_round(int mode, float v) {
  if (mode == kBf16) return bf16_round(v);
  if (mode == kTf32) return tf32_round(v);
  return v;
}

}  // namespace

extern "C" {

int orc_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

float orc_bf16_round(float f) { return bf16_round(f); }

// ---------------------------------------------------------------------------
// pkt data generator (examples/train_linear.cu:41-76): std::mt19937(42),
// W ~ N(0, 2/(m+n)), x ~ N(0,1), target = W x + N(0, 0.01^2) with the
// initial W, all drawn from one engine in this order.
void orc_pkt_make_linear_data(int m, int n, int batch, float* W, float* x, float* target) {
  std::mt19937 rng(42);
  const float scale = std::sqrt(2.0f / float(m + n));
  std::normal_distribution<float> wdist(0.0f, scale);
  std::normal_distribution<float> xdist(0.0f, 1.0f);
  std::normal_distribution<float> noise(0.0f, 0.01f);
  for (int i = 0; i < m * n; ++i) W[i] = wdist(rng);
  for (int i = 0; i < batch * n; ++i) x[i] = xdist(rng);
  for (int b = 0; b < batch; ++b) {
    for (int i = 0; i < m; ++i) {
      float acc = 0.0f;
      for (int j = 0; j < n; ++j) acc += W[i * n + j] * x[b * n + j];
      target[b * m + i] = acc + noise(rng);
    }
  }
}

// host_mse (examples/train_linear.cu:78-86): float accumulation in index order.
float orc_pkt_host_mse(const float* y, const float* t, long long count) {
  float acc = 0.f;
  for (long long i = 0; i < count; ++i) {
    float d = y[i] - t[i];
    acc += d * d;
  }
  return acc / static_cast<float>(count);
}

// cpu_train_linear (examples/train_linear.cu:101-151), restated with the same
// loop nest and float accumulation order so that its output matches pkt's
// host loop bit for bit. W is updated in place; loss_curve gets `steps` values.
void orc_pkt_cpu_train_linear(float* W, const float* x, const float* target, int batch, int m,
                              int n, int steps, float lr, float* loss_curve) {
  std::vector<float> y(size_t(batch) * m), dy(size_t(batch) * m);
  for (int step = 0; step < steps; ++step) {
    for (int b = 0; b < batch; ++b) {
      for (int i = 0; i < m; ++i) {
        float acc = 0.f;
        for (int j = 0; j < n; ++j) acc += W[i * n + j] * x[b * n + j];
        y[size_t(b) * m + i] = acc;
      }
    }
    float loss = 0.f;
    const float scale = 2.0f / float(batch * m);
    for (int i = 0; i < batch * m; ++i) {
      float diff = y[i] - target[i];
      dy[i] = scale * diff;
      loss += diff * diff;
    }
    loss /= float(batch * m);
    if (loss_curve) loss_curve[step] = loss;
    for (int i = 0; i < m; ++i) {
      for (int j = 0; j < n; ++j) {
        float grad = 0.f;
        for (int b = 0; b < batch; ++b) grad += dy[size_t(b) * m + i] * x[size_t(b) * n + j];
        W[i * n + j] -= lr * grad;
      }
    }
  }
}

// Axpy op (include/ops/axpy.cuh:33-46) with single-rounding FMA, as compiled by nvcc.
void orc_axpy(const float* x, float* y, float a, long long n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; ++i) y[i] = std::fmaf(a, x[i], y[i]);
}

// SGDUpdate op (include/ops/sgd.cuh:33-44): W[i] -= lr*dW[i]; nvcc contracts to
// fmaf(-lr, dW, W).
void orc_sgd(float* W, const float* dW, float lr, long long n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; ++i) W[i] = std::fmaf(-lr, dW[i], W[i]);
}

// ---------------------------------------------------------------------------
// MLP training step, the multi-layer extension of cpu_train_linear.
//
//   layers l = 0..L-1, W_l [d_{l+1}, d_l] row-major, b_l [d_{l+1}]
//   H_0 = x;  P_l = H_l W_l^T + b_l;  H_{l+1} = relu(P_l) for l < L-1;  Y = P_{L-1}
//   loss = sum (Y - t)^2 / (B d_L);  dY_{L-1} = 2 (Y - t) / (B d_L)
//   dW_l = dY_l^T H_l;  db_l = sum_b dY_l;  dY_{l-1} = (dY_l W_l) * [H_l > 0]
//   W_l -= lr dW_l;  b_l -= lr db_l
//
// mode 0 (fp32): fp64 accumulation of fp32 operands (the "truth").
// mode 1 (tf32): GEMM operands rounded to TF32 (nearest even), fp64 accumulation, fp32 storage.
// mode 2 (bf16): x, target, H, dY and the weight copy used by the GEMMs are
//   stored as bf16; GEMMs accumulate in fp64 here (fp32 on the GPU); fp32
//   master weights and fp32 bias.
// relu_last: apply ReLU to the output layer too (0 for every BASELINE config).
//
// W: concatenated layer weights (updated in place), b: concatenated biases or
// null (no bias). losses[steps]. If grads_dW / grads_db are non-null, the
// gradients of the LAST step are written there (same concatenated layout).
// If acts is non-null it receives H_1..H_{L-1} then Y of the last step's
// forward pass (concatenated, [B, d] each).
int orc_mlp_train(int L, const int* dims, int batch, int mode, int relu_last, const float* x,
                  const float* target, float* W, float* b, float lr, int steps, float* losses,
                  float* grads_dW, float* grads_db, float* acts) {
  if (L <= 0 || batch <= 0 || steps < 0) return -1;
  std::vector<size_t> woff(L + 1, 0), boff(L + 1, 0);
  for (int l = 0; l < L; ++l) {
    woff[l + 1] = woff[l] + size_t(dims[l + 1]) * dims[l];
    boff[l + 1] = boff[l] + size_t(dims[l + 1]);
  }
  const int dout = dims[L];
  std::vector<std::vector<float>> H(L + 1);  // H[0] = x (rounded), H[l] activations
  H[0].resize(size_t(batch) * dims[0]);
  for (size_t i = 0; i < H[0].size(); ++i) H[0][i] = store_round(mode, x[i]);
  std::vector<float> tq(size_t(batch) * dout);
  for (size_t i = 0; i < tq.size(); ++i) tq[i] = store_round(mode, target[i]);
  for (int l = 1; l <= L; ++l) H[l].resize(size_t(batch) * dims[l]);
  std::vector<float> Wop(woff[L]);
  std::vector<float> dYa, dYb;
  std::vector<float> dW, db;

  for (int step = 0; step < steps; ++step) {
    for (size_t i = 0; i < Wop.size(); ++i) Wop[i] = operand_round(mode, W[i]);
    // ---- forward
    for (int l = 0; l < L; ++l) {
      const int din = dims[l], dn = dims[l + 1];
      const float* Wl = Wop.data() + woff[l];
      const float* bl = b ? b + boff[l] : nullptr;
      const bool relu = (l < L - 1) || relu_last;
      const bool last = (l == L - 1);
      const std::vector<float>& Hin = H[l];
      std::vector<float>& Hout = H[l + 1];
#pragma omp parallel
      {
        std::vector<float> arow(din);
#pragma omp for schedule(static)
        for (int r = 0; r < batch; ++r) {
          for (int k = 0; k < din; ++k) arow[k] = operand_round(mode, Hin[size_t(r) * din + k]);
          for (int j = 0; j < dn; ++j) {
            const float* w = Wl + size_t(j) * din;
            double acc = 0.0;
            for (int k = 0; k < din; ++k) acc += double(arow[k]) * double(w[k]);
            float p = float(acc);
            if (bl) p = p + bl[j];
            if (relu && p < 0.f) p = 0.f;
            Hout[size_t(r) * dn + j] = last ? p : store_round(mode, p);
          }
        }
      }
    }
    // ---- loss + dY
    const std::vector<float>& Y = H[L];
    const double inv = 1.0 / (double(batch) * double(dout));
    const float scale = float(2.0 * inv);
    dYa.assign(size_t(batch) * dout, 0.f);
    double loss = 0.0;
#pragma omp parallel for reduction(+ : loss) schedule(static)
    for (long long i = 0; i < (long long)batch * dout; ++i) {
      float diff = Y[i] - tq[i];
      loss += double(diff) * double(diff);
      float g = scale * diff;
      if (relu_last && Y[i] <= 0.f) g = 0.f;
      dYa[i] = store_round(mode, g);
    }
    if (losses) losses[step] = float(loss * inv);
    if (acts && step == steps - 1) {
      size_t o = 0;
      for (int l = 1; l <= L; ++l) {
        std::memcpy(acts + o, H[l].data(), H[l].size() * 4);
        o += H[l].size();
      }
    }
    // ---- backward
    dW.assign(woff[L], 0.f);
    db.assign(boff[L], 0.f);
    for (int l = L - 1; l >= 0; --l) {
      const int din = dims[l], dn = dims[l + 1];
      const float* Wl = Wop.data() + woff[l];
      std::vector<float> dYop(dYa.size());
      for (size_t i = 0; i < dYa.size(); ++i) dYop[i] = operand_round(mode, dYa[i]);
      std::vector<float> Hop(H[l].size());
      for (size_t i = 0; i < Hop.size(); ++i) Hop[i] = operand_round(mode, H[l][i]);
      // wgrad: dW[j,k] = sum_b dY[b,j] H[b,k]
      float* dWl = dW.data() + woff[l];
#pragma omp parallel
      {
        std::vector<double> acc(din);
#pragma omp for schedule(static)
        for (int j = 0; j < dn; ++j) {
          std::fill(acc.begin(), acc.end(), 0.0);
          for (int r = 0; r < batch; ++r) {
            const double g = dYop[size_t(r) * dn + j];
            if (g == 0.0) continue;
            const float* h = Hop.data() + size_t(r) * din;
            for (int k = 0; k < din; ++k) acc[k] += g * double(h[k]);
          }
          for (int k = 0; k < din; ++k) dWl[size_t(j) * din + k] = float(acc[k]);
        }
      }
      if (b) {
        float* dbl = db.data() + boff[l];
#pragma omp parallel for schedule(static)
        for (int j = 0; j < dn; ++j) {
          double s = 0.0;
          for (int r = 0; r < batch; ++r) s += double(dYa[size_t(r) * dn + j]);
          dbl[j] = float(s);
        }
      }
      if (l > 0) {
        // dgrad: dH[b,k] = sum_j dY[b,j] W[j,k], masked by H_l > 0 (ReLU of layer l-1)
        dYb.assign(size_t(batch) * din, 0.f);
#pragma omp parallel
        {
          std::vector<double> acc(din);
#pragma omp for schedule(static)
          for (int r = 0; r < batch; ++r) {
            std::fill(acc.begin(), acc.end(), 0.0);
            for (int j = 0; j < dn; ++j) {
              const double g = dYop[size_t(r) * dn + j];
              if (g == 0.0) continue;
              const float* w = Wl + size_t(j) * din;
              for (int k = 0; k < din; ++k) acc[k] += g * double(w[k]);
            }
            for (int k = 0; k < din; ++k) {
              float v = float(acc[k]);
              if (!(H[l][size_t(r) * din + k] > 0.f)) v = 0.f;
              dYb[size_t(r) * din + k] = store_round(mode, v);
            }
          }
        }
        dYa.swap(dYb);
      }
    }
    // ---- SGD (fused multiply-add, as the GPU epilogue computes it)
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)woff[L]; ++i) W[i] = std::fmaf(-lr, dW[i], W[i]);
    if (b) {
      for (size_t i = 0; i < boff[L]; ++i) b[i] = std::fmaf(-lr, db[i], b[i]);
    }
    if (step == steps - 1) {
      if (grads_dW) std::memcpy(grads_dW, dW.data(), dW.size() * 4);
      if (grads_db && b) std::memcpy(grads_db, db.data(), db.size() * 4);
    }
  }
  return 0;
}

// Seeded data for the single-Linear train_linear configuration of the
// benchmark plan: std::mt19937(seed); x ~ N(0,1) [batch,in]; W ~ U(+-1/sqrt(in));
// b = 0; W*, b* ~ N(0,1); target = x W*^T + b* + N(0, noise^2).
void orc_make_linear_task(int in, int out, int batch, unsigned seed, float noise, float* x,
                          float* W, float* b, float* target) {
  std::mt19937 rng(seed);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  const float bound = 1.0f / std::sqrt(float(in));
  std::uniform_real_distribution<float> ud(-bound, bound);
  for (long long i = 0; i < (long long)batch * in; ++i) x[i] = nd(rng);
  for (long long i = 0; i < (long long)out * in; ++i) W[i] = ud(rng);
  for (int i = 0; i < out; ++i) b[i] = 0.0f;
  std::vector<float> Ws(size_t(out) * in), bs(out);
  for (auto& v : Ws) v = nd(rng);
  for (auto& v : bs) v = nd(rng);
  std::normal_distribution<float> nz(0.0f, noise);
  for (int r = 0; r < batch; ++r) {
    for (int j = 0; j < out; ++j) {
      double acc = 0.0;
      for (int k = 0; k < in; ++k) acc += double(x[size_t(r) * in + k]) * Ws[size_t(j) * in + k];
      target[size_t(r) * out + j] = float(acc) + bs[j] + nz(rng);
    }
  }
}

}  // extern "C"
