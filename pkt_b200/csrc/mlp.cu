// MLP training engine: the multi-layer generalisation of pkt's train_linear
// (examples/train_linear.cu:482-607 builds one Linear's forward / MSE /
// backward / SGD task DAG). Here one training step is ONE persistent launch of
// a tile-granular DAG:
//
//   FWD(l, i, j)   tcgen05 tile of H_{l+1} = act(H_l W_l^T + b_l), row block i
//                  waits on F[l-1][i] (all column tiles of row block i of the
//                  previous layer); the last layer's epilogue is MSE: it writes
//                  dY = 2(y-t)/(B n), per-tile loss partials and column sums of dY
//   LOSS_REDUCE    deterministic sum of the loss partials -> losses[step]
//   DGRAD(l, i, j) tile of dY_{l-1} = (dY_l W_l) * [H_l > 0], waits on row block i of dY_l
//   WGRAD(l, p, q) tile of dW_l = dY_l^T H_l (K = batch) with SGD fused into the
//                  epilogue (fp32 master update + bf16 copy for the next step),
//                  waits on all of dY_l
//   BIAS_SGD(l)    b_l -= lr * (sum of dY_l column partials)
//
// Weights the GEMMs read are double-buffered by step parity (bf16 copies, or
// the fp32 masters in TF32 mode), so the fused SGD of step s never races the
// forward / dgrad reads of step s.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/pk/detail/internal.h"
#include "runtime_impl.h"

namespace pkb {

namespace {

__global__ void f32_to_bf16_2d(const float* src, int rows, int cols, int lds, uint16_t* dst,
                               int ldd) {
  const long long total = (long long)rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = int(i / cols), c = int(i % cols);
    const float f = src[(long long)r * lds + c];
    uint16_t h;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(f));
    dst[(long long)r * ldd + c] = h;
  }
}

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Training steps one launch runs when pkt_mlp_train is asked for that many or
// more (grad_mode 0; even, so the weight parity after the launch is the one
// before it).
constexpr int kMultiSteps = 4;



// grad_mode 2: copies the fp32 master rows/cols of one weight tile from its
// owner's exchange region (a peer mapping) into this rank's copy.
__global__ void gather_master_tile(const float* src, float* dst, int rows, int cols, int ld) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)rows * cols;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols, c = i % cols;
    dst[r * ld + c] = src[r * ld + c];
  }
}

}  // namespace

struct Mlp {
  Runtime* rt = nullptr;
  int L = 0, B = 0;
  std::vector<int> dims, ld;
  bool bf = true;  // bf16 mode (else tf32)
  int es = 2;      // storage bytes per activation element
  bool has_bias = true, relu_last = false;
  float lr = 1e-3f;
  int grad_mode = 0;
  int max_bn = 256;
  float grad_scale = 1.0f;
  bool capture_y = false;

  // Two input slots (x, target): pkt_mlp_load_batch fills the idle slot and makes it
  // the active one, so the copy of the next batch can overlap the current step.
  void* Xs[2] = {nullptr, nullptr};
  void* Ts[2] = {nullptr, nullptr};
  int active_slot = 0;
  int next_slot = 0;
  std::vector<void*> H;   // H[l], l = 1..L-1 (index 0 unused)
  std::vector<void*> dY;  // dY[l], l = 0..L-1
  std::vector<float*> W32[2];
  std::vector<uint16_t*> Wbf[2];
  std::vector<float*> bias;
  std::vector<float*> colsum;
  float* loss_partials = nullptr;
  float* losses = nullptr;
  int* step_ctr = nullptr;
  int loss_cap = 1 << 16;
  int losses_enqueued = 0;
  float* Yout = nullptr;
  float* grads = nullptr;  // grad_mode 1: per layer one bucket [dW_l, db_l], layer 0 first
  long long grad_count = 0;
  std::vector<long long> dW_off, db_off;

  int parity = 0;
  int P = 2;    // CTA pair (cta_group::2, 256-row tiles) or single CTA (128-row tiles)
  int TM = 0;   // row tiles of the batch-row GEMMs: ceil(B / (128 P))
  int TMr = 0;  // 128-row blocks of the batch (TM * P): rows of the column / loss partials
  // step task lists by [weight parity][input slot]; update lists by weight parity
  std::vector<pkt_task> tasks[2][2], update[2];
  pkt_task* d_tasks[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};
  // kMultiSteps consecutive steps in one launch (grad_mode 0), by starting weight
  // parity and input slot; empty when not built
  std::vector<pkt_task> multi[2][2];
  pkt_task* d_multi[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};
  int wg_token_base = 0;  // token of layer 0's weight-gradient tiles (layer l: + l)
  pkt_task* d_update[2] = {nullptr, nullptr};
  // grad_mode 1: the step list split into L backward segments (segment s ends
  // with layer L-1-s's gradient complete), by weight parity and input slot;
  // seg_begin[p][q][s] is the first task of segment s (L + 1 entries)
  std::vector<pkt_task> segs[2][2];
  std::vector<int> seg_begin[2][2];
  pkt_task* d_segs[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};
  int reserved_sms = 0;  // SMs the persistent grid leaves free (for a collective on another stream)
  int num_tokens = 0;
  int gemm_tiles_per_step = 0;
  double flops_per_step = 0;

  // ---- fused data parallel (grad_mode 2): the exchange region holds the fp32
  // masters, both bf16 weight copies, the partial-tile slots, the bias
  // gradient vectors and the counters; peers map it through CUDA IPC.
  uint8_t* region = nullptr;
  size_t region_bytes = 0;
  std::vector<long long> master_off, wbf_off[2];
  std::vector<int> wg_tm, wg_tn, wg_bn, wg_base, bias_off;
  int wg_total = 0, bias_total = 0;
  pkb::DpPeers hdp{};
  pkb::DpPeers* d_dp = nullptr;
  int dp_world = 0, dp_rank = 0;  // dp_world 0: not connected yet
  uint8_t* peer_open[PKT_DP_MAX_RANKS] = {};
  int dp_step = 0;

  ~Mlp() {
    if (rt) cudaSetDevice(rt->device);
    auto F = [](void* p) { cudaFree(p); };
    for (int k = 0; k < 2; ++k) {
      F(Xs[k]);
      F(Ts[k]);
      F(d_tasks[k][0]);
      F(d_tasks[k][1]);
      F(d_multi[k][0]);
      F(d_multi[k][1]);
      F(d_segs[k][0]);
      F(d_segs[k][1]);
    }
    for (auto p : H) F(p);
    for (auto p : dY) F(p);
    if (region) {  // weights were carved from the exchange region
      for (int k = 0; k < 2; ++k) {
        W32[k].clear();
        Wbf[k].clear();
      }
      for (auto p : peer_open)
        if (p) cudaIpcCloseMemHandle(p);
      F(region);
      F(d_dp);
    }
    for (int k = 0; k < 2; ++k) {
      for (auto p : W32[k]) F(p);
      for (auto p : Wbf[k]) F(p);
      F(d_update[k]);
    }
    for (auto p : bias) F(p);
    for (auto p : colsum) F(p);
    F(loss_partials);
    F(losses);
    F(step_ctr);
    F(Yout);
    F(grads);
    delete rt;
  }

  int act_dtype() const { return bf ? PKT_DTYPE_BF16 : PKT_DTYPE_F32; }
  int in_dtype() const { return bf ? PKT_DTYPE_BF16 : PKT_DTYPE_TF32; }
  const void* Hin(int l, int q) const { return l == 0 ? Xs[q] : H[l]; }
  // weight copy the GEMMs of parity p read
  const void* Wop(int l, int p) const { return bf ? (const void*)Wbf[p][l] : (const void*)W32[p][l]; }
  float* Wmaster(int l, int p) const { return bf ? W32[0][l] : W32[p][l]; }

  int pick_bn(int M, int N, bool b_mn) const {
    // each CTA of a pair holds bn/P rows of B: a multiple of the 128-byte MN atom
    // (MN-major) or of 16 (K-major)
    const int align = (b_mn ? (bf ? 64 : 32) : 16) * P;
    int cap = std::min(max_bn, kMaxBN);
    int need = round_up(N, align);
    int bn = std::min(cap, need);
    bn = std::max(align, bn / align * align);
    const int tiles_m = (M + kBM * P - 1) / (kBM * P);
    // Narrower tiles only for GEMMs too small to give half of the CTAs (pairs) a
    // tile: the step's other GEMMs fill the rest, while a narrower tile has a
    // shorter k-block, which the stage ring (sized in bytes for the widest tile)
    // covers for less time, so its MMAs stall on loads.
    const int units = std::max(1, rt->num_sms / P);
    while (bn > std::max(64 * P, align) && 2LL * tiles_m * ((N + bn - 1) / bn) < units) {
      const int nb = bn / 2;
      if (nb % align != 0) break;
      bn = nb;
    }
    return bn;
  }

  // Tile width of layer l's weight-gradient GEMM.
  int wgrad_bn(int l) const { return pick_bn(dims[l + 1], dims[l], true); }

  int alloc(void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, std::max<size_t>(bytes, 16));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(mlp buffer)");
    cudaMemset(*p, 0, std::max<size_t>(bytes, 16));
    return PKT_OK;
  }

  int setup(const pkt_mlp_config& c);
  int build_multi();
  int setup_dp();
  int connect(int rank, int world, const uint8_t* handles);
  int build(int p, int q);
  int launch_list(pkt_task* d, int n, cudaStream_t st);
};

int Mlp::setup(const pkt_mlp_config& c) {
  L = c.num_layers;
  B = c.batch;
  if (L <= 0 || B <= 0 || !c.dims) return fail(PKT_ERR_ARGS, "bad MLP config");
  dims.assign(c.dims, c.dims + L + 1);
  for (int d : dims)
    if (d <= 0) return fail(PKT_ERR_ARGS, "layer widths must be positive");
  if (c.dtype != PKT_DTYPE_BF16 && c.dtype != PKT_DTYPE_TF32) return fail(PKT_ERR_ARGS, "dtype must be bf16 or tf32");
  bf = c.dtype == PKT_DTYPE_BF16;
  es = bf ? 2 : 4;
  has_bias = c.has_bias != 0;
  relu_last = c.relu_last != 0;
  lr = c.lr;
  grad_mode = c.grad_mode;
  max_bn = c.max_bn > 0 ? c.max_bn : 256;
  if (grad_mode < 0 || grad_mode > 2) return fail(PKT_ERR_ARGS, "grad_mode must be 0, 1 or 2");
  if (grad_mode == 2 && c.dtype != PKT_DTYPE_BF16)
    return fail(PKT_ERR_UNSUPPORTED, "fused data parallel (grad_mode 2) needs bf16 weights");
  ld.resize(L + 1);
  for (int l = 0; l <= L; ++l) ld[l] = round_up(dims[l], 64);
  if (c.cta_pair == 1 || c.cta_pair == 2) {
    P = c.cta_pair;
  } else {
    // Automatic: CTA pairs (256-row tiles, half the operand traffic per SM) when
    // the widest layer alone gives every pair a 256 x 256 tile; single CTAs
    // otherwise -- a narrow network is bound by the latency of its layer chain,
    // which a pair lengthens (both CTAs' loads land before the MMA starts, and
    // the pair hands its completion over before publishing it).
    long long widest = 0;
    for (int l = 0; l < L; ++l)
      widest = std::max(widest, (long long)((B + 255) / 256) * ((dims[l + 1] + 255) / 256));
    P = widest >= rt->num_sms / 2 ? 2 : 1;
  }
  TM = (B + kBM * P - 1) / (kBM * P);
  TMr = TM * P;
  int rc;
  for (int k = 0; k < 2; ++k) {
    if ((rc = alloc(&Xs[k], size_t(B) * ld[0] * es))) return rc;
    if ((rc = alloc(&Ts[k], size_t(B) * ld[L] * es))) return rc;
  }
  H.assign(L, nullptr);
  for (int l = 1; l < L; ++l)
    if ((rc = alloc(&H[l], size_t(B) * ld[l] * es))) return rc;
  dY.assign(L, nullptr);
  for (int l = 0; l < L; ++l)
    if ((rc = alloc(&dY[l], size_t(B) * ld[l + 1] * es))) return rc;
  for (int k = 0; k < 2; ++k) {
    W32[k].assign(L, nullptr);
    Wbf[k].assign(L, nullptr);
  }
  if (grad_mode == 2 && (rc = setup_dp())) return rc;
  for (int l = 0; l < L && grad_mode != 2; ++l) {
    const size_t n = size_t(dims[l + 1]) * ld[l];
    if ((rc = alloc((void**)&W32[0][l], n * 4))) return rc;
    if (!bf && (rc = alloc((void**)&W32[1][l], n * 4))) return rc;
    if (bf) {
      for (int k = 0; k < 2; ++k)
        if ((rc = alloc((void**)&Wbf[k][l], n * 2))) return rc;
    }
  }
  bias.assign(L, nullptr);
  colsum.assign(L, nullptr);
  for (int l = 0; l < L; ++l) {
    if ((rc = alloc((void**)&bias[l], size_t(ld[l + 1]) * 4))) return rc;
    if (has_bias && (rc = alloc((void**)&colsum[l], size_t(TMr) * ld[l + 1] * 4))) return rc;
  }
  if ((rc = alloc((void**)&loss_partials, size_t(TMr) * 64 * 4 + size_t(TMr) * ((dims[L] + 15) / 16) * 4))) return rc;
  if ((rc = alloc((void**)&losses, size_t(loss_cap) * 4))) return rc;
  if ((rc = alloc((void**)&step_ctr, 16))) return rc;
  if ((rc = alloc((void**)&Yout, size_t(B) * ld[L] * 4))) return rc;
  if (grad_mode == 1) {
    dW_off.resize(L);
    db_off.resize(L);
    long long o = 0;
    for (int l = 0; l < L; ++l) {  // contiguous per layer: one all-reduce bucket each
      dW_off[l] = o;
      o += (long long)dims[l + 1] * ld[l];
      db_off[l] = o;
      o += round_up(dims[l + 1], 4);
    }
    grad_count = o;
    if ((rc = alloc((void**)&grads, size_t(o) * 4))) return rc;
  }
  for (int l = 0; l < L; ++l) flops_per_step += 2.0 * B * dims[l] * dims[l + 1] * (l > 0 ? 3 : 2);
  return PKT_OK;
}

// Lays out and allocates the exchange region (grad_mode 2). Its size does not
// depend on the world size: a rank owns ceil(T / world) of the T weight tiles
// and keeps world partial slots for each, at most T + world - 1 slots.
int Mlp::setup_dp() {
  const int S = PKT_DP_MAX_RANKS;
  auto a256 = [](long long x) { return (x + 255) / 256 * 256; };
  wg_tm.assign(L, 0);
  wg_tn.assign(L, 0);
  wg_bn.assign(L, 0);
  wg_base.assign(L, 0);
  bias_off.assign(L, 0);
  wg_total = 0;
  bias_total = 0;
  for (int l = 0; l < L; ++l) {
    const int M = dims[l + 1], N = dims[l];
    wg_bn[l] = wgrad_bn(l);
    wg_tm[l] = (M + kBM * P - 1) / (kBM * P);
    wg_tn[l] = (N + wg_bn[l] - 1) / wg_bn[l];
    wg_base[l] = wg_total;
    wg_total += wg_tm[l] * wg_tn[l];
    bias_off[l] = bias_total;
    bias_total += round_up(dims[l + 1], 4);
  }
  long long off = 0;
  master_off.assign(L, 0);
  wbf_off[0].assign(L, 0);
  wbf_off[1].assign(L, 0);
  for (int l = 0; l < L; ++l) {
    const long long n = (long long)dims[l + 1] * ld[l];
    master_off[l] = off;
    off += a256(n * 4);
    for (int k = 0; k < 2; ++k) {
      wbf_off[k][l] = off;
      off += a256(n * 2);
    }
  }
  hdp = DpPeers{};
  hdp.pair = P;
  hdp.num_layers = L;
  hdp.slot_bytes = (long long)P * kBM * 256 * 4;
  hdp.recv_off = off;
  off += (long long)(wg_total + S) * hdp.slot_bytes;
  hdp.arrive_off = off;
  off += a256((long long)(wg_total + S) * 4);
  hdp.wready_off = off;
  off += a256((long long)L * 4);
  hdp.barrive_off = off;
  off += a256((long long)L * 4);
  hdp.bias_recv_off = off;
  hdp.bias_total = bias_total;
  off += a256((long long)2 * S * bias_total * 4);
  region_bytes = size_t(off);
  int rc = alloc((void**)&region, region_bytes);  // zeroed: counters start at 0
  if (rc) return rc;
  for (int k = 0; k < 2; ++k) {
    W32[k].assign(L, nullptr);
    Wbf[k].assign(L, nullptr);
  }
  for (int l = 0; l < L; ++l) {
    W32[0][l] = reinterpret_cast<float*>(region + master_off[l]);
    for (int k = 0; k < 2; ++k) Wbf[k][l] = reinterpret_cast<uint16_t*>(region + wbf_off[k][l]);
  }
  return PKT_OK;
}

int Mlp::connect(int rank, int world, const uint8_t* handles) {
  if (grad_mode != 2) return fail(PKT_ERR_ARGS, "pkt_mlp_dp_connect needs grad_mode 2");
  if (dp_world != 0) return fail(PKT_ERR_ARGS, "already connected");
  if (world < 1 || world > PKT_DP_MAX_RANKS || rank < 0 || rank >= world)
    return fail(PKT_ERR_ARGS, "rank %d / world %d out of range (world <= %d)", rank, world, PKT_DP_MAX_RANKS);
  if (world > 1 && handles == nullptr) return fail(PKT_ERR_ARGS, "peer handles missing");
  for (int r = 0; r < world; ++r) {
    if (r == rank) {
      hdp.base[r] = region;
      continue;
    }
    cudaIpcMemHandle_t hd;
    std::memcpy(&hd, handles + size_t(r) * sizeof(cudaIpcMemHandle_t), sizeof(hd));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, hd, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle(peer exchange region)");
    peer_open[r] = static_cast<uint8_t*>(ptr);
    hdp.base[r] = peer_open[r];
  }
  hdp.world = world;
  hdp.rank = rank;
  const long long slot_rows = (long long)P * kBM, nslots = wg_total + PKT_DP_MAX_RANKS;
  for (int r = 0; r < world; ++r)
    if (!make_store_map(&hdp.recv_map[r], hdp.base[r] + hdp.recv_off, PKT_DTYPE_F32, 256,
                        nslots * slot_rows, 256))
      return fail(PKT_ERR_CUDA, "tensor map over rank %d's partial slots", r);
  cudaError_t e = cudaMalloc(&d_dp, sizeof(DpPeers));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(peer table)");
  e = cudaMemcpy(d_dp, &hdp, sizeof(DpPeers), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "copy peer table");
  dp_world = world;
  dp_rank = rank;
  return PKT_OK;
}

// Registers the GEMMs of weight parity p and input slot q and builds their task lists.
int Mlp::build(int p, int q) {
  const int cur = p, nxt = 1 - p;
  std::vector<pkt_gemm_desc> g;
  std::vector<int> fwd(L), dgr(L, -1), wgr(L);
  // ---- forward
  for (int l = 0; l < L; ++l) {
    pkt_gemm_desc d{};
    d.M = B;
    d.N = dims[l + 1];
    d.K = dims[l];
    d.in_dtype = in_dtype();
    d.a = Hin(l, q);
    d.lda = ld[l];
    d.a_major = PKT_MAJOR_K;
    d.b = Wop(l, cur);
    d.ldb = ld[l];
    d.b_major = PKT_MAJOR_K;
    d.bn = pick_bn(d.M, d.N, false);
    d.bias = has_bias ? bias[l] : nullptr;
    if (l < L - 1) {
      d.epilogue = PKT_EPI_BIAS_ACT;
      d.relu = 1;
      d.out = H[l + 1];
      d.ldo = ld[l + 1];
      d.out_dtype = act_dtype();
    } else {
      d.epilogue = PKT_EPI_MSE;
      d.relu = relu_last ? 1 : 0;
      d.out = dY[L - 1];
      d.ldo = ld[L];
      d.out_dtype = act_dtype();
      d.aux = Ts[q];
      d.ldaux = ld[L];
      d.scale = float(2.0 / (double(B) * double(dims[L])));
      d.loss_partials = loss_partials;
      d.colsum = has_bias ? colsum[L - 1] : nullptr;
      d.ldcol = ld[L];
      d.y_out = capture_y ? Yout : nullptr;
      d.ldy = ld[L];
    }
    fwd[l] = int(g.size());
    d.cta_pair = P;
    g.push_back(d);
  }
  // ---- dgrad (l >= 1) and wgrad
  for (int l = L - 1; l >= 0; --l) {
    if (l >= 1) {
      pkt_gemm_desc d{};
      d.M = B;
      d.N = dims[l];
      d.K = dims[l + 1];
      d.in_dtype = in_dtype();
      d.a = dY[l];
      d.lda = ld[l + 1];
      d.a_major = PKT_MAJOR_K;
      d.b = Wop(l, cur);
      d.ldb = ld[l];
      d.b_major = PKT_MAJOR_MN;
      d.bn = pick_bn(d.M, d.N, true);
      d.epilogue = PKT_EPI_DGRAD_RELU;
      d.out = dY[l - 1];
      d.ldo = ld[l];
      d.out_dtype = act_dtype();
      d.aux = H[l];
      d.ldaux = ld[l];
      d.colsum = has_bias ? colsum[l - 1] : nullptr;
      d.ldcol = ld[l];
      dgr[l] = int(g.size());
      d.cta_pair = P;
    g.push_back(d);
    }
    pkt_gemm_desc d{};
    d.M = dims[l + 1];
    d.N = dims[l];
    d.K = B;
    d.in_dtype = in_dtype();
    d.a = dY[l];
    d.lda = ld[l + 1];
    d.a_major = PKT_MAJOR_MN;
    d.b = Hin(l, q);
    d.ldb = ld[l];
    d.b_major = PKT_MAJOR_MN;
    d.bn = wgrad_bn(l);
    if (grad_mode == 2) {
      // the owner of a tile applies SGD to its master shard and writes the bf16
      // copy the next step reads (locally here, on the other ranks in the kernel)
      d.epilogue = PKT_EPI_WGRAD_PEER;
      d.w_in = Wmaster(l, cur);
      d.w_out = Wmaster(l, nxt);
      d.w_shadow = Wbf[nxt][l];
      d.ldw = ld[l];
      d.lr = lr * grad_scale;
      d.out = nullptr;
    } else if (grad_mode == 0) {
      d.epilogue = PKT_EPI_WGRAD_SGD;
      d.w_in = Wmaster(l, cur);
      d.w_out = Wmaster(l, nxt);
      d.w_shadow = bf ? (void*)Wbf[nxt][l] : nullptr;
      d.ldw = ld[l];
      d.lr = lr;
      d.out = nullptr;
    } else {
      d.epilogue = PKT_EPI_WGRAD_STORE;
      d.out = grads + dW_off[l];
      d.ldo = ld[l];
      d.out_dtype = PKT_DTYPE_F32;
    }
    wgr[l] = int(g.size());
    d.cta_pair = P;
    g.push_back(d);
  }
  int first = 0;
  int rc = rt->register_gemms(g.data(), int(g.size()), &first);
  if (rc) return rc;
  auto G = [&](int idx) -> const DevGemm& { return rt->host_gemms[first + idx]; };
  if (grad_mode == 2) {
    // weight-gradient tiles are numbered across layers: tile t goes to rank t % world
    for (int l = 0; l < L; ++l) {
      DevGemm& dg = rt->host_gemms[first + wgr[l]];
      if (dg.tiles_m != wg_tm[l] || dg.tiles_n != wg_tn[l] || dg.d.bn != wg_bn[l])
        return fail(PKT_ERR_UNSUPPORTED, "weight tile layout differs from the exchange region's");
      dg.dp_tile_base = wg_base[l];
      dg.dp_layer = l;
      cudaError_t e = cudaMemcpy(rt->d_gemms + first + wgr[l], &dg, sizeof(DevGemm), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return cuda_fail(e, "copy gemm table");
    }
  }

  // ---- tokens
  int next_id = 1;
  std::vector<std::vector<int>> F(L, std::vector<int>(TM)), Bk(L, std::vector<int>(TM));
  std::vector<int> BF(L);
  for (int l = 0; l < L; ++l)
    for (int i = 0; i < TM; ++i) F[l][i] = next_id++;
  for (int l = 0; l < L - 1; ++l)
    for (int i = 0; i < TM; ++i) Bk[l][i] = next_id++;
  for (int i = 0; i < TM; ++i) Bk[L - 1][i] = F[L - 1][i];
  for (int l = 0; l < L; ++l) BF[l] = next_id++;
  const int WG_base = next_id;
  wg_token_base = WG_base;
  next_id += L;
  std::vector<int> WR(L, 0);  // grad_mode 2: this step's weights of layer l have arrived
  if (grad_mode == 2)
    for (int l = 0; l < L; ++l) WR[l] = next_id++;
  num_tokens = next_id;
  if (num_tokens > 65535) return fail(PKT_ERR_UNSUPPORTED, "too many dependency tokens");
  // marks per row block of dY_l (and total)
  std::vector<int> dy_tn(L);
  for (int l = 0; l < L; ++l) dy_tn[l] = (l == L - 1) ? G(fwd[L - 1]).tiles_n : G(dgr[l + 1]).tiles_n;

  std::vector<pkt_task>& tl = tasks[p][q];
  tl.clear();
  auto gemm_task = [&](int gidx, int i, int j) {
    pkt_task t{};
    t.header.opcode = PKT_OP_GEMM;
    pkt_gemm_tile_args a{uint32_t(first + gidx), uint32_t(i), uint32_t(j), 0};
    t.header.arg_bytes = sizeof(a);
    std::memcpy(t.args, &a, sizeof(a));
    return t;
  };
  int tiles = 0;
  if (grad_mode == 2) {
    for (int l = 0; l < L; ++l) {
      pkt_task t{};
      t.header.opcode = PKT_OP_DP_WAIT;
      pkt_dp_wait_args a{l, wg_tm[l] * wg_tn[l]};
      t.header.arg_bytes = sizeof(a);
      std::memcpy(t.args, &a, sizeof(a));
      t.header.buffer_write_id = uint16_t(WR[l]);
      tl.push_back(t);
    }
  }
  // Forward: layer by layer, row block by row block. (Listing the layers as an
  // interleaved wavefront was measured slower: a row block's input has to be
  // complete when it is dequeued, and with every controller running up to
  // kSlots tasks ahead of its pipeline that needs hundreds of tiles of distance
  // in the list, which leaves little to interleave.)
  for (int l = 0; l < L; ++l) {
    const DevGemm& dg = G(fwd[l]);
    for (int i = 0; i < TM; ++i)
      for (int j = 0; j < dg.tiles_n; ++j) {
        pkt_task t = gemm_task(fwd[l], i, j);
        if (l > 0) {
          t.header.buffer_read_id = uint16_t(F[l - 1][i]);
          t.header.wait_count = uint32_t(G(fwd[l - 1]).tiles_n);
        }
        t.header.buffer_write_id = uint16_t(F[l][i]);
        if (l == L - 1) t.header.ext_ids = uint32_t(BF[L - 1]) << 16;
        if (grad_mode == 2) {  // second read: the layer's weights of this step
          t.header.ext_ids |= uint32_t(WR[l]);
          t.header.ext_wait_count = 1;
        }
        tl.push_back(t);
        ++tiles;
      }
  }
  if (grad_mode != 2) {
    // The dgrad chain (the critical path) first, layer by layer, row block by
    // row block. The last layer's weight-gradient tiles need only the complete
    // dY_{L-1}, which the forward's last tiles finish: they are spread over the
    // dgrad tiles, from a distance of four grid waves after the forward on (long
    // K = batch mainloops between the short ones of a K = d_L dgrad layer, whose
    // epilogues would otherwise hold the MMA issuer). The other layers' weight-
    // gradient tiles, which need a complete dY_l, follow the whole dgrad chain:
    // by the time a CTA dequeues them their inputs are normally complete.
    auto wgrad_order = [&](int l) {
      const DevGemm& wg = G(wgr[l]);
      // groups of 8 tile rows swept column by column: the tiles in flight share
      // fewer operand blocks, so more of them stay in L2
      std::vector<std::pair<int, int>> order;
      for (int i0 = 0; i0 < wg.tiles_m; i0 += 8)
        for (int j = 0; j < wg.tiles_n; ++j)
          for (int i = i0; i < std::min(wg.tiles_m, i0 + 8); ++i) order.push_back({i, j});
      return order;
    };
    auto emit_wgrad = [&](int l, int i, int j) {
      pkt_task t = gemm_task(wgr[l], i, j);
      t.header.buffer_read_id = uint16_t(BF[l]);
      t.header.wait_count = uint32_t(TM * dy_tn[l]);
      t.header.buffer_write_id = uint16_t(WG_base + l);
      tl.push_back(t);
      ++tiles;
    };
    auto emit_dgrad = [&](int l, int i) {
      const DevGemm& dg = G(dgr[l]);
      for (int j = 0; j < dg.tiles_n; ++j) {
        pkt_task t = gemm_task(dgr[l], i, j);
        t.header.buffer_read_id = uint16_t(Bk[l][i]);
        t.header.wait_count = uint32_t(dy_tn[l]);
        t.header.buffer_write_id = uint16_t(Bk[l - 1][i]);
        t.header.ext_ids = uint32_t(BF[l - 1]) << 16;
        tl.push_back(t);
        ++tiles;
      }
    };
    const std::vector<std::pair<int, int>> wlast = wgrad_order(L - 1);
    size_t wnext = 0;
    long long dgrad_tiles = 0, dgrad_listed = 0;
    for (int l = L - 1; l >= 1; --l) dgrad_tiles += (long long)TM * G(dgr[l]).tiles_n;
    const int units = std::max(1, rt->num_sms / P);
    const long long start = 4LL * units;
    // A layer whose weight gradient is only a few tiles (a narrow, latency-bound
    // network) has them listed right after its dgrad tiles instead: dY_l is then
    // complete or nearly so, the few CTAs that take them wait at most one layer,
    // and the weight gradients overlap the rest of the dgrad chain instead of
    // following it.
    auto small_wgrad = [&](int l) { return G(wgr[l]).tiles_m * G(wgr[l]).tiles_n * 2 <= units; };
    std::vector<char> wg_done(L, 0);
    for (int l = L - 1; l >= 1; --l) {
      for (int i = 0; i < TM; ++i) {
        emit_dgrad(l, i);
        dgrad_listed += G(dgr[l]).tiles_n;
        if (small_wgrad(L - 1) || dgrad_listed < start || dgrad_tiles <= start) continue;
        const long long want = (long long)wlast.size() * (dgrad_listed - start) / (dgrad_tiles - start);
        for (; (long long)wnext < want && wnext < wlast.size(); ++wnext)
          emit_wgrad(L - 1, wlast[wnext].first, wlast[wnext].second);
      }
      if (small_wgrad(l)) {
        for (const auto& ij : wgrad_order(l)) emit_wgrad(l, ij.first, ij.second);
        wg_done[l] = 1;
      }
    }
    for (int l = L - 1; l >= 0; --l) {
      const std::vector<std::pair<int, int>> order = wgrad_order(l);
      for (size_t k = (l == L - 1 ? wnext : 0); k < order.size() && !wg_done[l]; ++k)
        emit_wgrad(l, order[k].first, order[k].second);
      if (has_bias) {
        const int n = dims[l + 1];
        for (int c0 = 0; c0 < n; c0 += 512) {
          pkt_task t{};
          t.header.opcode = PKT_OP_BIAS_SGD;
          pkt_bias_sgd_args a{};
          a.partials = colsum[l];
          a.num_partials = TMr;
          a.ld = ld[l + 1];
          a.col_begin = c0;
          a.col_end = std::min(n, c0 + 512);
          if (grad_mode == 0) {
            a.bias = bias[l];
            a.lr = lr;
          } else {
            a.grad_out = grads + db_off[l];
          }
          t.header.arg_bytes = sizeof(a);
          std::memcpy(t.args, &a, sizeof(a));
          t.header.buffer_read_id = uint16_t(BF[l]);
          t.header.wait_count = uint32_t(TM * dy_tn[l]);
          tl.push_back(t);
        }
      }
    }
  } else {
    // Fused data parallel: each layer's weight-gradient tiles follow its dgrad
    // tiles, so partial tiles cross to their owners (and the owners' new
    // weights back) while the rest of the backward runs. A weight-gradient
    // epilogue only sends its partial; the owner's reduce task of a tile (sum,
    // SGD, new bf16 tile to every rank) is listed after the next layer's whole
    // dgrad block (layer 1's after layer 0's weight-gradient tiles, layer 0's
    // last): a weight-gradient tile of the wide layers runs ~75 us, and a reduce
    // dequeued before the ranks' partials have landed holds its CTA pair
    // waiting (listed two dgrad waves later, the reduces averaged 57 us each on
    // two GPUs, mostly waiting). No GEMM epilogue ever waits on another rank.
    const float lre = lr * grad_scale;
    std::vector<pkt_task> deferred;  // this rank's reduce tasks of the previous layer
    std::vector<pkt_task> last;      // layer 0's reduce tasks
    for (int l = L - 1; l >= 0; --l) {
      if (l >= 1) {
        const DevGemm& dg = G(dgr[l]);
        for (int i = 0; i < TM; ++i)
          for (int j = 0; j < dg.tiles_n; ++j) {
            pkt_task t = gemm_task(dgr[l], i, j);
            t.header.buffer_read_id = uint16_t(Bk[l][i]);
            t.header.wait_count = uint32_t(dy_tn[l]);
            t.header.buffer_write_id = uint16_t(Bk[l - 1][i]);
            t.header.ext_ids = uint32_t(BF[l - 1]) << 16;
            tl.push_back(t);
            ++tiles;
          }
        for (auto& d2 : deferred) tl.push_back(d2);
        deferred.clear();
      }
      // weight-gradient tiles grouped by owner, starting with the next rank's
      // (this rank's own last): the ranks' partials of a tile leave at different
      // times, so the owners' slots fill evenly
      const DevGemm& wg = G(wgr[l]);
      const int world = dp_world > 0 ? dp_world : 1, me = dp_world > 0 ? dp_rank : 0;
      for (int k = 1; k <= world; ++k) {
        const int owner = (me + k) % world;
        for (int i = 0; i < wg.tiles_m; ++i)
          for (int j = 0; j < wg.tiles_n; ++j) {
            if ((wg_base[l] + i * wg.tiles_n + j) % world != owner) continue;
            pkt_task t = gemm_task(wgr[l], i, j);
            t.header.buffer_read_id = uint16_t(BF[l]);
            t.header.wait_count = uint32_t(TM * dy_tn[l]);
            tl.push_back(t);
            ++tiles;
            if (owner == me) {
              pkt_task r = gemm_task(wgr[l], i, j);
              r.header.opcode = PKT_OP_DP_REDUCE;
              (l >= 1 ? deferred : last).push_back(r);
            }
          }
      }
      if (l == 0) {  // no dgrad block follows: layer 1's reduce tasks go here
        for (auto& d2 : deferred) tl.push_back(d2);
        deferred.clear();
      }
      if (has_bias) {
        pkt_task t{};
        t.header.opcode = PKT_OP_DP_BIAS_SEND;
        pkt_dp_bias_args a{};
        a.partials = colsum[l];
        a.num_partials = TMr;
        a.ld = ld[l + 1];
        a.n = dims[l + 1];
        a.layer = l;
        a.bias_off = bias_off[l];
        t.header.arg_bytes = sizeof(a);
        std::memcpy(t.args, &a, sizeof(a));
        t.header.buffer_read_id = uint16_t(BF[l]);
        t.header.wait_count = uint32_t(TM * dy_tn[l]);
        tl.push_back(t);
      }
    }
    for (auto& r : last) tl.push_back(r);
    if (has_bias) {
      for (int l = L - 1; l >= 0; --l) {
        pkt_task t{};
        t.header.opcode = PKT_OP_DP_BIAS_APPLY;
        pkt_dp_bias_args a{};
        a.bias = bias[l];
        a.n = dims[l + 1];
        a.layer = l;
        a.bias_off = bias_off[l];
        a.lr = lre;
        t.header.arg_bytes = sizeof(a);
        std::memcpy(t.args, &a, sizeof(a));
        t.header.buffer_read_id = uint16_t(BF[l]);
        t.header.wait_count = uint32_t(TM * dy_tn[l]);
        tl.push_back(t);
      }
    }
  }
  {
    // last in the list: the MSE tiles it sums finished long before, so it never
    // holds a CTA waiting
    const DevGemm& dg = G(fwd[L - 1]);
    pkt_task t{};
    t.header.opcode = PKT_OP_LOSS_REDUCE;
    pkt_loss_reduce_args a{loss_partials, losses, dg.tiles_m * P * dg.tiles_n,
                           float(1.0 / (double(B) * double(dims[L]))), step_ctr};
    t.header.arg_bytes = sizeof(a);
    std::memcpy(t.args, &a, sizeof(a));
    t.header.buffer_read_id = uint16_t(BF[L - 1]);
    t.header.wait_count = uint32_t(TM * dg.tiles_n);
    tl.push_back(t);
  }
  gemm_tiles_per_step = tiles;

  // ---- separate update list (grad_mode 1): runs after the gradient all-reduce
  std::vector<pkt_task>& ul = update[p];
  ul.clear();
  if (grad_mode == 1) {
    const float lre = lr * grad_scale;
    for (int l = 0; l < L; ++l) {
      const long long n = (long long)dims[l + 1] * ld[l];
      const long long chunk = 1 << 16;
      for (long long o = 0; o < n; o += chunk) {
        pkt_task t{};
        t.header.opcode = PKT_OP_SGD_MIXED;
        pkt_sgd_mixed_args a{};
        a.w = Wmaster(l, cur) + o;
        a.g = grads + dW_off[l] + o;
        a.w_out = Wmaster(l, nxt) + o;
        a.w_bf16 = bf ? Wbf[nxt][l] + o : nullptr;
        a.n = std::min(chunk, n - o);
        a.lr = lre;
        t.header.arg_bytes = sizeof(a);
        std::memcpy(t.args, &a, sizeof(a));
        ul.push_back(t);
      }
      if (has_bias) {
        pkt_task t{};
        t.header.opcode = PKT_OP_BIAS_SGD;
        pkt_bias_sgd_args a{};
        a.partials = grads + db_off[l];
        a.num_partials = 1;
        a.ld = 0;
        a.col_begin = 0;
        a.col_end = dims[l + 1];
        a.bias = bias[l];
        a.lr = lre;
        t.header.arg_bytes = sizeof(a);
        std::memcpy(t.args, &a, sizeof(a));
        ul.push_back(t);
      }
    }
  }
  // ---- backward segments (grad_mode 1): the same tasks as the step list, in
  // its order, split into L launches so that a caller can all-reduce layer l's
  // gradient bucket on another stream while the following segments run (one
  // collective per layer, overlapped with the rest of the backward). Segment 0
  // holds the forward, the loss and layer L-1's weight / bias gradient; segment
  // s >= 1 the dgrad tiles that produce dY_l and layer l's gradient, l = L-1-s.
  // A launch starts with its tokens at zero, so every dependency count drops by
  // the publishes earlier segments made (complete: stream order) and a count
  // they already satisfied disappears.
  std::vector<pkt_task>& sl = segs[p][q];
  std::vector<int>& sb = seg_begin[p][q];
  sl.clear();
  sb.clear();
  if (grad_mode == 1) {
    auto seg_of = [&](const pkt_task& t) -> int {
      const uint16_t op = t.header.opcode;
      if (op == PKT_OP_GEMM) {
        pkt_gemm_tile_args a;
        std::memcpy(&a, t.args, sizeof(a));
        const int gi = int(a.gemm) - first;
        for (int l = 0; l < L; ++l) {
          if (gi == fwd[l]) return 0;
          if (gi == wgr[l]) return L - 1 - l;
          if (l >= 1 && gi == dgr[l]) return L - l;  // it produces dY_{l-1}
        }
        return -1;
      }
      if (op == PKT_OP_BIAS_SGD) {
        pkt_bias_sgd_args a;
        std::memcpy(&a, t.args, sizeof(a));
        for (int l = 0; l < L; ++l)
          if (a.partials == colsum[l]) return L - 1 - l;
        return -1;
      }
      if (op == PKT_OP_LOSS_REDUCE) return 0;
      return -1;
    };
    std::vector<int> seg(tl.size());
    std::vector<std::vector<int>> pub(L, std::vector<int>(num_tokens, 0));
    for (size_t i = 0; i < tl.size(); ++i) {
      seg[i] = seg_of(tl[i]);
      if (seg[i] < 0) return fail(PKT_ERR_UNSUPPORTED, "task %zu has no backward segment", i);
      const pkt_task_header& h = tl[i].header;
      if (h.read_epoch != 0) return fail(PKT_ERR_UNSUPPORTED, "segmented lists take no epochs");
      if (h.buffer_write_id) pub[seg[i]][h.buffer_write_id]++;
      if (h.ext_ids >> 16) pub[seg[i]][h.ext_ids >> 16]++;
    }
    // returns false when a count needs publishes of a later segment
    auto adjust = [&](int s, int tok, uint32_t need, int* id_out, uint32_t* need_out) {
      int before = 0;
      for (int k = 0; k < s; ++k) before += pub[k][tok];
      if (int(need) <= before) {
        *id_out = 0;
        *need_out = 0;
        return true;
      }
      *id_out = tok;
      *need_out = need - uint32_t(before);
      return int(*need_out) <= pub[s][tok];
    };
    for (int s = 0; s < L; ++s) {
      sb.push_back(int(sl.size()));
      for (size_t i = 0; i < tl.size(); ++i) {
        if (seg[i] != s) continue;
        pkt_task t = tl[i];
        pkt_task_header& h = t.header;
        int id = 0;
        uint32_t need = 0;
        if (h.buffer_read_id) {
          if (!adjust(s, h.buffer_read_id, h.wait_count, &id, &need))
            return fail(PKT_ERR_UNSUPPORTED, "task %zu waits for a later segment", i);
          h.buffer_read_id = uint16_t(id);
          h.wait_count = need;
        }
        if (h.ext_ids & 0xffffu) {
          if (!adjust(s, int(h.ext_ids & 0xffffu), h.ext_wait_count, &id, &need))
            return fail(PKT_ERR_UNSUPPORTED, "task %zu waits for a later segment", i);
          h.ext_ids = (h.ext_ids & 0xffff0000u) | uint32_t(id);
          h.ext_wait_count = need;
        }
        sl.push_back(t);
      }
    }
    sb.push_back(int(sl.size()));
  }
  // ---- device copies
  cudaFree(d_segs[p][q]);
  d_segs[p][q] = nullptr;
  if (!sl.empty()) {
    cudaError_t e = cudaMalloc(&d_segs[p][q], sizeof(pkt_task) * sl.size());
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(segment tasks)");
    e = cudaMemcpy(d_segs[p][q], sl.data(), sizeof(pkt_task) * sl.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "copy segment tasks");
  }
  cudaFree(d_tasks[p][q]);
  cudaFree(d_update[p]);
  d_tasks[p][q] = d_update[p] = nullptr;
  cudaError_t e = cudaMalloc(&d_tasks[p][q], sizeof(pkt_task) * std::max<size_t>(1, tl.size()));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(step tasks)");
  e = cudaMemcpy(d_tasks[p][q], tl.data(), sizeof(pkt_task) * tl.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "copy step tasks");
  if (!ul.empty()) {
    e = cudaMalloc(&d_update[p], sizeof(pkt_task) * ul.size());
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(update tasks)");
    e = cudaMemcpy(d_update[p], ul.data(), sizeof(pkt_task) * ul.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "copy update tasks");
  }
  return rt->ensure_tokens(num_tokens);
}

// kMultiSteps steps in one launch (grad_mode 0): the single-step lists of
// alternating weight parity, each step on its own range of dependency tokens.
// Every weight-gradient tile, bias-update and loss-reduce task of a step also
// counts on one "step done" token, which the next step's first-layer forward
// tiles read. That covers every task of the step: the weight-gradient tiles need
// every dgrad tile (dY_0 needs the whole dgrad chain) and every forward tile
// (dY_{L-1} needs the whole forward) -- so the next step neither reads weights
// before their update nor overwrites activations, gradients or loss partials the
// step still reads. It saves the launch, the token reset and the ramp-up /
// drain of the persistent grid between steps.
int Mlp::build_multi() {
  for (int p = 0; p < 2; ++p)
    for (int q = 0; q < 2; ++q) {
      multi[p][q].clear();
      cudaFree(d_multi[p][q]);
      d_multi[p][q] = nullptr;
    }
  if (grad_mode != 0) return PKT_OK;
  const int T = num_tokens + 1;  // tokens per step: the step's own plus its "step done"
  if ((long long)kMultiSteps * T > 65535) return PKT_OK;  // single-step launches only
  for (int p = 0; p < 2; ++p)
    for (int q = 0; q < 2; ++q) {
      std::vector<pkt_task>& ml = multi[p][q];
      int done_count = 0;  // tasks of one step that count on its "step done" token
      for (int k = 0; k < kMultiSteps; ++k) {
        const std::vector<pkt_task>& one = tasks[(p + k) & 1][q];
        const int off = k * T, done = off + num_tokens;
        int count = 0;
        auto shift = [&](uint32_t id) { return id == 0 ? 0u : id + uint32_t(off); };
        for (const pkt_task& t0 : one) {
          pkt_task t = t0;
          pkt_task_header& h = t.header;
          const bool wgrad = h.opcode == PKT_OP_GEMM && h.buffer_write_id >= wg_token_base &&
                             h.buffer_write_id < wg_token_base + L;
          h.buffer_read_id = uint16_t(shift(h.buffer_read_id));
          h.buffer_write_id = uint16_t(shift(h.buffer_write_id));
          h.ext_ids = shift(h.ext_ids & 0xffffu) | (shift(h.ext_ids >> 16) << 16);
          if (wgrad) {  // the per-layer token nothing else reads becomes the step's
            h.buffer_write_id = uint16_t(done);
            ++count;
          } else if ((h.opcode == PKT_OP_BIAS_SGD || h.opcode == PKT_OP_LOSS_REDUCE) &&
                     h.buffer_write_id == 0) {
            h.buffer_write_id = uint16_t(done);
            ++count;
          }
          if (k > 0 && h.opcode == PKT_OP_GEMM && h.buffer_read_id == 0) {
            // a first-layer forward tile: after the whole previous step
            h.buffer_read_id = uint16_t(done - T);
            h.wait_count = uint32_t(done_count);
          }
          ml.push_back(t);
        }
        done_count = count;
      }
      cudaError_t e = cudaMalloc(&d_multi[p][q], sizeof(pkt_task) * ml.size());
      if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(multi-step tasks)");
      e = cudaMemcpy(d_multi[p][q], ml.data(), sizeof(pkt_task) * ml.size(), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return cuda_fail(e, "copy multi-step tasks");
    }
  return rt->ensure_tokens(kMultiSteps * T);
}

int Mlp::launch_list(pkt_task* d, int n, cudaStream_t st) {
  rt->num_tokens = rt->token_cap;
  cudaError_t e = cudaMemsetAsync(rt->d_state, 0, sizeof(int) * state_ints(rt->num_tokens), st);
  if (e != cudaSuccess) return cuda_fail(e, "reset token state");
  KParams kp{};
  kp.tasks = d;
  kp.num_tasks = n;
  kp.num_tokens = rt->num_tokens;
  kp.state = rt->d_state;
  kp.gemms = rt->d_gemms;
  kp.num_gemms = rt->num_gemms;
  kp.chunk = 1;
  kp.timeout_ns = rt->timeout_ns;
  kp.perf = nullptr;
  kp.dp = d_dp;
  kp.dp_step = dp_step;
  // A controller dequeues its next task only when at most one (single CTAs) or
  // two (pairs) of its published tasks still wait for its epilogue warps: a
  // dependent tile a busy CTA dequeued early would wait behind that CTA's long
  // tiles while other CTAs idle. Measured against the slot ring alone: the
  // 16 x 512 network 0.345 -> 0.332 ms per step (1, single CTAs; 2 gives 0.344),
  // the ragged TF32 one 0.286 -> 0.261 ms (2, pairs); the 4096-wide one equal in
  // SM cycles.
  kp.lookahead = P == 1 ? 1 : 2;
  if (rt->perf_enabled) {
    if (rt->perf_cap < rt->num_sms) {
      cudaFree(rt->d_perf);
      e = cudaMalloc(&rt->d_perf, sizeof(unsigned long long) * PKT_PERF_WORDS * rt->num_sms);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(perf)");
      rt->perf_cap = rt->num_sms;
    }
    cudaMemsetAsync(rt->d_perf, 0, sizeof(unsigned long long) * PKT_PERF_WORDS * rt->perf_cap, st);
    kp.perf = rt->d_perf;
  }
  kp.clock_acc = rt->d_clock;
  int blocks = 0;
  int rc = rt->clamp_blocks(std::max(P, rt->num_sms - reserved_sms), P, &blocks);
  if (rc) return rc;
  rc = rt->trace_for(n, st, &kp.trace);
  if (rc) return rc;
  rt->last_blocks = blocks;
  e = launch_megakernel(kp, blocks, st, P);
  if (e != cudaSuccess) return cuda_fail(e, "launch megakernel");
  return PKT_OK;
}

}  // namespace pkb

using pkb::Mlp;
struct pkt_mlp {
  Mlp* m;
};

static int rebuild(Mlp* m) {
  m->rt->num_gemms = 0;
  m->rt->host_gemms.clear();
  for (int p = 0; p < 2; ++p)
    for (int q = 0; q < 2; ++q) {
      int rc = m->build(p, q);
      if (rc) return rc;
    }
  return m->build_multi();
}

extern "C" {

int pkt_mlp_create(int device, const pkt_mlp_config* cfg, pkt_mlp** out) {
  if (!cfg || !out) return pkb::fail(PKT_ERR_ARGS, "null argument");
  pkb::Runtime* rt = nullptr;
  int rc = pkb::Runtime::create(device, &rt);
  if (rc) return rc;
  Mlp* m = new Mlp();
  m->rt = rt;
  rc = m->setup(*cfg);
  if (!rc) rc = rebuild(m);
  if (rc) {
    delete m;
    return rc;
  }
  *out = new pkt_mlp{m};
  return PKT_OK;
}

int pkt_mlp_destroy(pkt_mlp* h) {
  if (!h) return PKT_OK;
  delete h->m;
  delete h;
  return PKT_OK;
}

int pkt_mlp_set_params(pkt_mlp* h, const float* W, const float* b) {
  if (!h || !W) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  cudaSetDevice(m->rt->device);
  cudaDeviceSynchronize();
  size_t wo = 0, bo = 0;
  for (int l = 0; l < m->L; ++l) {
    const int rows = m->dims[l + 1], cols = m->dims[l];
    float* dst = m->Wmaster(l, m->parity);
    cudaError_t e = cudaMemcpy2D(dst, size_t(m->ld[l]) * 4, W + wo, size_t(cols) * 4, size_t(cols) * 4, rows,
                                 cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return pkb::cuda_fail(e, "copy weights");
    if (m->bf) {
      pkb::f32_to_bf16_2d<<<256, 256>>>(dst, rows, cols, m->ld[l], m->Wbf[m->parity][l], m->ld[l]);
    }
    wo += size_t(rows) * cols;
    if (b) {
      e = cudaMemcpy(m->bias[l], b + bo, size_t(rows) * 4, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return pkb::cuda_fail(e, "copy bias");
    } else {
      cudaMemset(m->bias[l], 0, size_t(rows) * 4);
    }
    bo += rows;
  }
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return pkb::cuda_fail(e, "set params");
  return PKT_OK;
}

int pkt_mlp_get_params(pkt_mlp* h, float* W, float* b) {
  if (!h || !W) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  cudaSetDevice(m->rt->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return pkb::cuda_fail(e, "sync");
  if (m->grad_mode == 2 && m->dp_world > 1) {
    // each rank updated only the master tiles it owns: fetch the others from
    // their owners (every rank must have finished the same steps)
    const int rows_t = pkb::kBM * m->P;
    for (int l = 0; l < m->L; ++l)
      for (int i = 0; i < m->wg_tm[l]; ++i)
        for (int j = 0; j < m->wg_tn[l]; ++j) {
          const int t = m->wg_base[l] + i * m->wg_tn[l] + j, owner = t % m->dp_world;
          if (owner == m->dp_rank) continue;
          const long long el = (long long)i * rows_t * m->ld[l] + (long long)j * m->wg_bn[l];
          const float* src = reinterpret_cast<const float*>(m->hdp.base[owner] + m->master_off[l]) + el;
          float* dst = reinterpret_cast<float*>(m->region + m->master_off[l]) + el;
          pkb::gather_master_tile<<<64, 256>>>(src, dst, std::min(rows_t, m->dims[l + 1] - i * rows_t),
                                               std::min(m->wg_bn[l], m->dims[l] - j * m->wg_bn[l]), m->ld[l]);
        }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return pkb::cuda_fail(e, "gather master shards");
  }
  size_t wo = 0, bo = 0;
  for (int l = 0; l < m->L; ++l) {
    const int rows = m->dims[l + 1], cols = m->dims[l];
    e = cudaMemcpy2D(W + wo, size_t(cols) * 4, m->Wmaster(l, m->parity), size_t(m->ld[l]) * 4, size_t(cols) * 4,
                     rows, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return pkb::cuda_fail(e, "read weights");
    wo += size_t(rows) * cols;
    if (b) {
      e = cudaMemcpy(b + bo, m->bias[l], size_t(rows) * 4, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) return pkb::cuda_fail(e, "read bias");
    }
    bo += rows;
  }
  return PKT_OK;
}

int pkt_mlp_get_grads(pkt_mlp* h, float* dW, float* db) {
  if (!h || !dW) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  if (m->grad_mode != 1) return pkb::fail(PKT_ERR_ARGS, "gradients are only stored with grad_mode 1");
  cudaSetDevice(m->rt->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return pkb::cuda_fail(e, "sync");
  size_t wo = 0, bo = 0;
  for (int l = 0; l < m->L; ++l) {
    const int rows = m->dims[l + 1], cols = m->dims[l];
    e = cudaMemcpy2D(dW + wo, size_t(cols) * 4, m->grads + m->dW_off[l], size_t(m->ld[l]) * 4, size_t(cols) * 4,
                     rows, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return pkb::cuda_fail(e, "read grads");
    wo += size_t(rows) * cols;
    if (db) {
      e = cudaMemcpy(db + bo, m->grads + m->db_off[l], size_t(rows) * 4, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) return pkb::cuda_fail(e, "read bias grads");
    }
    bo += rows;
  }
  return PKT_OK;
}

int pkt_mlp_load_batch(pkt_mlp* h, const void* x, const void* t, int on_device, void* stream) {
  if (!h || !x || !t) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  cudaSetDevice(m->rt->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const int q = m->next_slot;
  // One linear copy per tensor when the device rows are unpadded (the common
  // case: widths that are multiples of 64); a pitched copy only for padded rows.
  auto copy_rows = [&](void* dst, const void* src, int width) -> cudaError_t {
    const size_t row = size_t(width) * m->es;
    const size_t pitch = size_t(pkb::round_up(width, 64)) * m->es;
    if (pitch == row) return cudaMemcpyAsync(dst, src, row * m->B, kind, st);
    return cudaMemcpy2DAsync(dst, pitch, src, row, row, m->B, kind, st);
  };
  cudaError_t e = copy_rows(m->Xs[q], x, m->dims[0]);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "copy x");
  e = copy_rows(m->Ts[q], t, m->dims[m->L]);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "copy target");
  m->active_slot = q;
  m->next_slot = q ^ 1;
  return PKT_OK;
}

int pkt_mlp_train(pkt_mlp* h, int steps, void* stream) {
  if (!h || steps < 0) return pkb::fail(PKT_ERR_ARGS, "bad argument");
  Mlp* m = h->m;
  if (m->losses_enqueued + steps > m->loss_cap)
    return pkb::fail(PKT_ERR_ARGS, "loss buffer full (%d steps); call pkt_mlp_reset_losses", m->loss_cap);
  cudaSetDevice(m->rt->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (m->grad_mode == 2 && m->dp_world == 0)
    return pkb::fail(PKT_ERR_ARGS, "grad_mode 2: call pkt_mlp_dp_connect before training");
  for (int s = 0; s < steps;) {
    const int p = m->parity, q = m->active_slot;
    if (steps - s >= pkb::kMultiSteps && m->d_multi[p][q]) {
      int rc = m->launch_list(m->d_multi[p][q], int(m->multi[p][q].size()), st);
      if (rc) return rc;
      s += pkb::kMultiSteps;
      m->losses_enqueued += pkb::kMultiSteps;
      continue;  // kMultiSteps is even: the parity is unchanged
    }
    ++s;
    int rc = m->launch_list(m->d_tasks[p][q], int(m->tasks[p][q].size()), st);
    if (rc) return rc;
    if (m->grad_mode == 2) m->dp_step++;
    if (m->grad_mode == 1) {
      rc = m->launch_list(m->d_update[p], int(m->update[p].size()), st);
      if (rc) return rc;
    }
    m->parity ^= 1;
    m->losses_enqueued++;
  }
  return PKT_OK;
}

int pkt_mlp_forward_backward(pkt_mlp* h, void* stream) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  if (m->grad_mode != 1) return pkb::fail(PKT_ERR_ARGS, "forward_backward needs grad_mode 1");
  if (m->losses_enqueued + 1 > m->loss_cap) return pkb::fail(PKT_ERR_ARGS, "loss buffer full");
  cudaSetDevice(m->rt->device);
  m->losses_enqueued++;
  const int p = m->parity, q = m->active_slot;
  return m->launch_list(m->d_tasks[p][q], int(m->tasks[p][q].size()), static_cast<cudaStream_t>(stream));
}

int pkt_mlp_apply_update(pkt_mlp* h, void* stream) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  if (m->grad_mode != 1) return pkb::fail(PKT_ERR_ARGS, "apply_update needs grad_mode 1");
  cudaSetDevice(m->rt->device);
  const int p = m->parity;
  int rc = m->launch_list(m->d_update[p], int(m->update[p].size()), static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  m->parity ^= 1;
  return PKT_OK;
}

int pkt_mlp_backward_segments(pkt_mlp* h, int* count) {
  if (!h || !count) return pkb::fail(PKT_ERR_ARGS, "null argument");
  if (h->m->grad_mode != 1) return pkb::fail(PKT_ERR_ARGS, "backward segments exist with grad_mode 1 only");
  *count = h->m->L;
  return PKT_OK;
}

int pkt_mlp_forward_backward_segment(pkt_mlp* h, int segment, void* stream) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  if (m->grad_mode != 1) return pkb::fail(PKT_ERR_ARGS, "backward segments exist with grad_mode 1 only");
  if (segment < 0 || segment >= m->L) return pkb::fail(PKT_ERR_ARGS, "segment %d of %d", segment, m->L);
  const int p = m->parity, q = m->active_slot;
  const std::vector<int>& sb = m->seg_begin[p][q];
  if (int(sb.size()) != m->L + 1) return pkb::fail(PKT_ERR_ARGS, "segments not built");
  if (segment == 0) {
    if (m->losses_enqueued + 1 > m->loss_cap) return pkb::fail(PKT_ERR_ARGS, "loss buffer full");
    m->losses_enqueued++;
  }
  cudaSetDevice(m->rt->device);
  return m->launch_list(m->d_segs[p][q] + sb[segment], sb[segment + 1] - sb[segment],
                        static_cast<cudaStream_t>(stream));
}

int pkt_mlp_grad_bucket(pkt_mlp* h, int layer, long long* offset, long long* count) {
  if (!h || !offset || !count) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  if (m->grad_mode != 1) return pkb::fail(PKT_ERR_ARGS, "gradient buffer exists with grad_mode 1 only");
  if (layer < 0 || layer >= m->L) return pkb::fail(PKT_ERR_ARGS, "layer %d of %d", layer, m->L);
  *offset = m->dW_off[layer];
  *count = (layer + 1 < m->L ? m->dW_off[layer + 1] : m->grad_count) - m->dW_off[layer];
  return PKT_OK;
}

int pkt_mlp_set_reserved_sms(pkt_mlp* h, int sms) {
  if (!h || sms < 0) return pkb::fail(PKT_ERR_ARGS, "bad argument");
  if (sms > h->m->rt->num_sms - 2) return pkb::fail(PKT_ERR_ARGS, "the grid needs at least 2 SMs");
  h->m->reserved_sms = sms;
  return PKT_OK;
}

int pkt_mlp_grad_buffer(pkt_mlp* h, float** ptr, long long* count) {
  if (!h || !ptr || !count) return pkb::fail(PKT_ERR_ARGS, "null argument");
  if (h->m->grad_mode != 1) return pkb::fail(PKT_ERR_ARGS, "gradient buffer exists with grad_mode 1 only");
  *ptr = h->m->grads;
  *count = h->m->grad_count;
  return PKT_OK;
}

int pkt_mlp_dp_handle(pkt_mlp* h, void* handle64) {
  if (!h || !handle64) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  if (m->grad_mode != 2 || !m->region) return pkb::fail(PKT_ERR_ARGS, "pkt_mlp_dp_handle needs grad_mode 2");
  cudaSetDevice(m->rt->device);
  cudaIpcMemHandle_t hd;
  cudaError_t e = cudaIpcGetMemHandle(&hd, m->region);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "cudaIpcGetMemHandle(exchange region)");
  std::memcpy(handle64, &hd, sizeof(hd));
  return PKT_OK;
}

int pkt_mlp_dp_connect(pkt_mlp* h, int rank, int world, const void* handles) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  cudaSetDevice(m->rt->device);
  cudaDeviceSynchronize();
  int rc = m->connect(rank, world, static_cast<const uint8_t*>(handles));
  if (rc) return rc;
  return rebuild(m);  // task lists depend on which tiles this rank owns
}

int pkt_mlp_set_grad_scale(pkt_mlp* h, float scale) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  cudaSetDevice(h->m->rt->device);
  cudaDeviceSynchronize();
  h->m->grad_scale = scale;
  return rebuild(h->m);
}

int pkt_mlp_set_output_capture(pkt_mlp* h, int enabled) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  cudaSetDevice(h->m->rt->device);
  cudaDeviceSynchronize();
  h->m->capture_y = enabled != 0;
  return rebuild(h->m);
}

int pkt_mlp_losses(pkt_mlp* h, float* out, int max_n, int* n) {
  if (!h || !out || !n) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  cudaSetDevice(m->rt->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return pkb::cuda_fail(e, "sync");
  const int k = std::min(max_n, m->losses_enqueued);
  if (k > 0) {
    e = cudaMemcpy(out, m->losses, sizeof(float) * k, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return pkb::cuda_fail(e, "read losses");
  }
  *n = k;
  return PKT_OK;
}

int pkt_mlp_reset_losses(pkt_mlp* h) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  cudaSetDevice(m->rt->device);
  cudaDeviceSynchronize();
  cudaMemset(m->step_ctr, 0, 16);
  m->losses_enqueued = 0;
  return PKT_OK;
}

int pkt_mlp_loss_ptr(pkt_mlp* h, int i, float** out) {
  if (!h || !out || i < 0 || i >= h->m->loss_cap) return pkb::fail(PKT_ERR_ARGS, "bad argument");
  *out = h->m->losses + i;
  return PKT_OK;
}

int pkt_mlp_get_output(pkt_mlp* h, float* y) {
  if (!h || !y) return pkb::fail(PKT_ERR_ARGS, "null argument");
  Mlp* m = h->m;
  if (!m->capture_y) return pkb::fail(PKT_ERR_ARGS, "output capture is off (pkt_mlp_set_output_capture)");
  cudaSetDevice(m->rt->device);
  cudaError_t e = cudaMemcpy2D(y, size_t(m->dims[m->L]) * 4, m->Yout, size_t(m->ld[m->L]) * 4,
                               size_t(m->dims[m->L]) * 4, m->B, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "read output");
  return PKT_OK;
}

int pkt_mlp_status(pkt_mlp* h, int* code, int* task_index, int* detail) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  return h->m->rt->status(code, task_index, detail);
}

int pkt_mlp_step_info(pkt_mlp* h, int* tasks, int* gemm_tiles, double* flops) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  if (tasks) *tasks = int(h->m->tasks[0][0].size() + h->m->update[0].size());
  if (gemm_tiles) *gemm_tiles = h->m->gemm_tiles_per_step;
  if (flops) *flops = h->m->flops_per_step;
  return PKT_OK;
}

}  // extern "C"

extern "C" {

int pkt_mlp_set_perf(pkt_mlp* h, int enabled) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  h->m->rt->perf_enabled = enabled != 0;
  return PKT_OK;
}

int pkt_mlp_set_trace(pkt_mlp* h, int enabled) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  h->m->rt->trace_enabled = enabled != 0;
  return PKT_OK;
}

int pkt_mlp_fetch_trace(pkt_mlp* h, unsigned long long* out, int max_tasks, int* n) {
  if (!h || !out || !n) return pkb::fail(PKT_ERR_ARGS, "null argument");
  return h->m->rt->fetch_trace(out, max_tasks, n);
}

int pkt_mlp_clock_stats(pkt_mlp* h, unsigned long long* out3, int reset) {
  if (!h) return pkb::fail(PKT_ERR_ARGS, "null argument");
  return h->m->rt->clock_stats(out3, reset != 0);
}

int pkt_mlp_fetch_perf(pkt_mlp* h, unsigned long long* out, int max_blocks, int* blocks) {
  if (!h || !out || !blocks) return pkb::fail(PKT_ERR_ARGS, "null argument");
  pkb::Runtime* rt = h->m->rt;
  if (!rt->perf_enabled || !rt->d_perf) return pkb::fail(PKT_ERR_ARGS, "perf counters are off");
  cudaSetDevice(rt->device);
  const int nb = std::min(max_blocks, rt->last_blocks);
  cudaError_t e = cudaMemcpy(out, rt->d_perf, sizeof(unsigned long long) * PKT_PERF_WORDS * nb,
                             cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "read perf");
  *blocks = nb;
  return PKT_OK;
}

}  // extern "C"
