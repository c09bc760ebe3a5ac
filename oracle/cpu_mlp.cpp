// Timed CPU baseline: pkt's host training loop in fp32, extended to the MLP and
// parallelised with OpenMP over the host cores.
//
// TEST / BENCHMARK INFRASTRUCTURE ONLY: loaded by bench.py's cpu_baseline leg and
// reference arm (and by tests/ to check it), never by the product path.
//
// What it restates: pkt's cpu_train_linear (examples/train_linear.cu:101-151) computes,
// per step, y = x W^T (fp32 accumulation), dy = 2 (y - t) / (B m) with the loss
// sum (y - t)^2 / (B m) (include/ops/mse.cuh:36-60), dW = dy^T x and W -= lr dW.
// Here the same fp32 arithmetic is extended with bias, ReLU on the hidden layers,
// dgrad through the ReLU mask and the bias gradient, for L layers:
//   H_0 = x;  H_{l+1} = relu(H_l W_l^T + b_l) (no ReLU on the output)
//   dY_{L-1} = 2 (Y - t) / (B d_L);  dW_l = dY_l^T H_l;  db_l = sum_b dY_l
//   dY_{l-1} = (dY_l W_l) * [H_l > 0];  W_l -= lr dW_l;  b_l -= lr db_l
// Every GEMM is written as rows of rank-1 updates C[i, :] += a[i, p] * B[p, :]
// (the forward uses W_l^T, transposed once per step), blocked for the caches and
// split over OpenMP threads, so the compiler's vectoriser (-O3 -march=native on the
// machine it runs on) emits FMA over the contiguous output row.
//
// Build: `make -C oracle native` (on the machine that runs it: -march=native).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// One vector register of floats: 16 with AVX-512, 8 otherwise (AVX2 / SSE split it).
#ifdef __AVX512F__
constexpr int kVW = 16;
#else
constexpr int kVW = 8;
#endif
typedef float v16 __attribute__((vector_size(kVW * 4)));
typedef float v16u __attribute__((vector_size(kVW * 4), aligned(4)));  // the same, unaligned in memory

constexpr int kRB = 6;    // rows per register block
constexpr int kCB = 4 * kVW;  // output columns per register block (4 vectors)
constexpr int kIB = 96;   // rows per cache block (reuse of a B panel)
constexpr int kPB = 256;  // reduction depth per cache block
constexpr int kJB = 512;  // output columns per cache block

// C[M, N] = A[M, K] * B[K, N]; row-major, leading dimensions lda / ldb / ldc.
// a_trans: A is given as At[K, M] (A[i, p] = At[p * lda + i]).
void gemm(int M, int N, int K, const float* A, int lda, bool a_trans, const float* B, int ldb,
          float* C, int ldc) {
  const int mb = (M + kIB - 1) / kIB, nb = (N + kJB - 1) / kJB;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int ib = 0; ib < mb; ++ib) {
    for (int jb = 0; jb < nb; ++jb) {
      const int iend = std::min(M, (ib + 1) * kIB), j0 = jb * kJB;
      const int jend = std::min(N, j0 + kJB);
      for (int p0 = 0; p0 < K; p0 += kPB) {
        const int pend = std::min(K, p0 + kPB);
        for (int c0 = j0; c0 < jend; c0 += kCB) {
          const int cols = std::min(kCB, jend - c0);
          for (int i0 = ib * kIB; i0 < iend; i0 += kRB) {
            const int rows = std::min(kRB, iend - i0);
            if (rows == kRB && cols == kCB) {
              // register block: kRB rows x 4 vectors of columns, all in registers
              v16 acc[kRB][4];
#pragma GCC unroll 8
              for (int r = 0; r < kRB; ++r)
#pragma GCC unroll 8
                for (int v = 0; v < 4; ++v)
                  acc[r][v] = p0 > 0 ? *reinterpret_cast<const v16u*>(C + size_t(i0 + r) * ldc + c0 + kVW * v)
                                     : v16{};
              for (int p = p0; p < pend; ++p) {
                const v16u* bp = reinterpret_cast<const v16u*>(B + size_t(p) * ldb + c0);
                const v16 b0 = bp[0], b1 = bp[1], b2 = bp[2], b3 = bp[3];
#pragma GCC unroll 8
                for (int r = 0; r < kRB; ++r) {
                  const float a = a_trans ? A[size_t(p) * lda + i0 + r] : A[size_t(i0 + r) * lda + p];
                  acc[r][0] += a * b0;
                  acc[r][1] += a * b1;
                  acc[r][2] += a * b2;
                  acc[r][3] += a * b3;
                }
              }
#pragma GCC unroll 8
              for (int r = 0; r < kRB; ++r)
#pragma GCC unroll 8
                for (int v = 0; v < 4; ++v)
                  *reinterpret_cast<v16u*>(C + size_t(i0 + r) * ldc + c0 + kVW * v) = acc[r][v];
              continue;
            }
            float acc[kRB][kCB];
            for (int r = 0; r < kRB; ++r)
              for (int c = 0; c < kCB; ++c)
                acc[r][c] = (r < rows && c < cols && p0 > 0) ? C[size_t(i0 + r) * ldc + c0 + c] : 0.f;
            for (int p = p0; p < pend; ++p) {
              const float* b = B + size_t(p) * ldb + c0;
              for (int r = 0; r < rows; ++r) {
                const float a = a_trans ? A[size_t(p) * lda + i0 + r] : A[size_t(i0 + r) * lda + p];
                for (int c = 0; c < cols; ++c) acc[r][c] += a * b[c];
              }
            }
            for (int r = 0; r < rows; ++r)
              for (int c = 0; c < cols; ++c) C[size_t(i0 + r) * ldc + c0 + c] = acc[r][c];
          }
        }
      }
    }
  }
}

void transpose(const float* src, int rows, int cols, float* dst) {
#pragma omp parallel for schedule(static)
  for (int c0 = 0; c0 < cols; c0 += 32)
    for (int r = 0; r < rows; ++r)
      for (int c = c0; c < std::min(cols, c0 + 32); ++c) dst[size_t(c) * rows + r] = src[size_t(r) * cols + c];
}

struct Ctx {
  int L = 0, B = 0;
  std::vector<int> dims;
  std::vector<std::vector<float>> H, WT, dW, db;
  std::vector<float> dYa, dYb;
};

}  // namespace

extern "C" {

int cpu_mlp_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void cpu_mlp_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

// Working buffers for one configuration (allocated and touched here, outside
// any timed region).
void* cpu_mlp_create(int L, const int* dims, int batch) {
  if (L <= 0 || batch <= 0) return nullptr;
  Ctx* c = new Ctx();
  c->L = L;
  c->B = batch;
  c->dims.assign(dims, dims + L + 1);
  c->H.resize(L + 1);
  for (int l = 1; l <= L; ++l) c->H[l].assign(size_t(batch) * dims[l], 0.f);
  c->WT.resize(L);
  c->dW.resize(L);
  c->db.resize(L);
  int wmax = 0;
  for (int l = 0; l < L; ++l) {
    c->WT[l].assign(size_t(dims[l]) * dims[l + 1], 0.f);
    c->dW[l].assign(size_t(dims[l]) * dims[l + 1], 0.f);
    c->db[l].assign(dims[l + 1], 0.f);
    wmax = std::max(wmax, dims[l + 1]);
  }
  c->dYa.assign(size_t(batch) * wmax, 0.f);
  c->dYb.assign(size_t(batch) * wmax, 0.f);
  return c;
}

void cpu_mlp_destroy(void* h) { delete static_cast<Ctx*>(h); }

// One training step on x [B, d_0], t [B, d_L]; W (concatenated [d_{l+1}, d_l]) and
// b (concatenated, or null) are updated in place; returns the step's loss.
float cpu_mlp_step(void* h, const float* x, const float* t, float* W, float* b, float lr) {
  Ctx& c = *static_cast<Ctx*>(h);
  const int L = c.L, B = c.B;
  const std::vector<int>& d = c.dims;
  std::vector<size_t> wo(L + 1, 0), bo(L + 1, 0);
  for (int l = 0; l < L; ++l) {
    wo[l + 1] = wo[l] + size_t(d[l + 1]) * d[l];
    bo[l + 1] = bo[l] + size_t(d[l + 1]);
  }
  // ---- forward
  for (int l = 0; l < L; ++l) {
    transpose(W + wo[l], d[l + 1], d[l], c.WT[l].data());
    const float* in = l == 0 ? x : c.H[l].data();
    float* out = c.H[l + 1].data();
    gemm(B, d[l + 1], d[l], in, d[l], false, c.WT[l].data(), d[l + 1], out, d[l + 1]);
    const bool relu = l < L - 1;
    const float* bl = b ? b + bo[l] : nullptr;
    const int n = d[l + 1];
#pragma omp parallel for schedule(static)
    for (int r = 0; r < B; ++r) {
      float* o = out + size_t(r) * n;
      for (int j = 0; j < n; ++j) {
        float v = o[j] + (bl ? bl[j] : 0.f);
        o[j] = (relu && v < 0.f) ? 0.f : v;
      }
    }
  }
  // ---- MSE (include/ops/mse.cuh:36-60 scaling)
  const int dout = d[L];
  const long long ny = (long long)B * dout;
  const float scale = 2.0f / float(ny);
  const float* Y = c.H[L].data();
  float* dY = c.dYa.data();
  double loss = 0.0;
#pragma omp parallel for reduction(+ : loss) schedule(static)
  for (long long i = 0; i < ny; ++i) {
    const float diff = Y[i] - t[i];
    loss += double(diff * diff);
    dY[i] = scale * diff;
  }
  // ---- backward
  for (int l = L - 1; l >= 0; --l) {
    const int din = d[l], dn = d[l + 1];
    const float* in = l == 0 ? x : c.H[l].data();
    dY = c.dYa.data();
    // dW_l = dY_l^T H_l  (A = dY^T given as dY [B, dn]: a_trans)
    gemm(dn, din, B, dY, dn, true, in, din, c.dW[l].data(), din);
    if (b) {
      float* g = c.db[l].data();
#pragma omp parallel for schedule(static)
      for (int j = 0; j < dn; ++j) {
        float s = 0.f;
        for (int r = 0; r < B; ++r) s += dY[size_t(r) * dn + j];
        g[j] = s;
      }
    }
    if (l > 0) {
      float* dprev = c.dYb.data();
      gemm(B, din, dn, dY, dn, false, W + wo[l], din, dprev, din);
      const float* Hl = c.H[l].data();
#pragma omp parallel for schedule(static)
      for (long long i = 0; i < (long long)B * din; ++i)
        if (!(Hl[i] > 0.f)) dprev[i] = 0.f;
      c.dYa.swap(c.dYb);
    }
  }
  // ---- SGD (include/ops/sgd.cuh:33-44)
  for (int l = 0; l < L; ++l) {
    float* w = W + wo[l];
    const float* g = c.dW[l].data();
    const long long n = (long long)d[l + 1] * d[l];
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < n; ++i) w[i] -= lr * g[i];
    if (b)
      for (int j = 0; j < d[l + 1]; ++j) b[bo[l] + j] -= lr * c.db[l][j];
  }
  return float(loss / double(ny));
}

}  // extern "C"
