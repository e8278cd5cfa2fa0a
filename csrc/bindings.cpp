// Python bindings of the sm_100a kernels (module hrm_flashrenderer_b200._C).
//
// Every entry point validates devices, dtypes, shapes, contiguity and alignment and launches on the current
// torch CUDA stream (so the calls are capturable in CUDA graphs).  Scratch memory (split-K partials, tickets,
// attention split partials) is passed in by the caller; nothing here allocates except the returned outputs of the
// convenience wrappers.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "gemm_w8a16.h"
#include "kernels.h"
#include "comm.h"

namespace py = pybind11;

namespace {

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_DTYPE(t, d) TORCH_CHECK((t).scalar_type() == (d), #t " has dtype ", (t).scalar_type(), ", expected ", (d))

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_ws(const hrm::GemmPlan& p, const at::Tensor& ws, const at::Tensor& counters) {
  if (p.ws_floats > 0) {
    CHECK_CUDA(ws);
    CHECK_CUDA(counters);
    CHECK_DTYPE(ws, at::kFloat);
    CHECK_DTYPE(counters, at::kInt);
    TORCH_CHECK((size_t)ws.numel() >= p.ws_floats, "split-K workspace too small: need ", p.ws_floats, " floats");
    TORCH_CHECK(counters.numel() >= p.counters, "split-K counters too small: need ", p.counters);
  }
}

hrm::GemmArgs base_args(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scale,
                        const c10::optional<at::Tensor>& bias, const at::Tensor& ws, const at::Tensor& counters,
                        const c10::optional<at::Tensor>& status = c10::nullopt) {
  CHECK_CUDA(x); CHECK_CUDA(w); CHECK_CUDA(scale);
  CHECK_DTYPE(x, at::kHalf); CHECK_DTYPE(w, at::kChar); CHECK_DTYPE(scale, at::kFloat);
  TORCH_CHECK(x.dim() == 2, "x [M,K] must be 2-D");
  TORCH_CHECK(x.stride(1) == 1, "x inner dim must be contiguous");
  hrm::GemmArgs a{};
  if (w.dim() == 3) {   // pre-tiled [ceil(N/128)][K/64][8192]
    TORCH_CHECK(w.is_contiguous() && w.size(2) == 8192, "tiled w must be contiguous [N/128, K/64, 8192]");
    TORCH_CHECK(w.size(1) * 64 == x.size(1), "K mismatch: x ", x.size(1), " vs tiled w ", w.size(1) * 64);
    TORCH_CHECK(w.size(0) == (scale.numel() + 127) / 128, "tiled w row tiles do not match scale (N entries)");
    a.N = (int)scale.numel();
    a.w_tiles = w.data_ptr<int8_t>();
  } else {
    TORCH_CHECK(w.dim() == 2 && w.stride(1) == 1, "w must be [N,K] with contiguous rows (or pre-tiled 3-D)");
    TORCH_CHECK(x.size(1) == w.size(1), "K mismatch: x ", x.size(1), " vs w ", w.size(1));
    TORCH_CHECK(w.stride(0) == w.size(1), "w must be row-major contiguous");
    TORCH_CHECK(scale.numel() == w.size(0), "scale must have N entries");
    a.N = (int)w.size(0);
  }
  a.M = (int)x.size(0);
  a.K = (int)x.size(1);
  a.scale = scale.data_ptr<float>();
  if (bias.has_value() && bias->defined()) {
    CHECK_DTYPE((*bias), at::kFloat);
    TORCH_CHECK(bias->numel() == a.N, "bias must have N entries");
    a.bias = bias->data_ptr<float>();
  }
  a.ws = ws.defined() && ws.numel() ? ws.data_ptr<float>() : nullptr;
  a.counters = counters.defined() && counters.numel() ? counters.data_ptr<int>() : nullptr;
  if (status.has_value() && status->defined()) {
    CHECK_DTYPE((*status), at::kInt);
    a.status = status->data_ptr<int>();
  }
  return a;
}

// (n_tile, m_tile, kt) of units [u0, u1) as the GEMM producer walks them, flattened; host-side check of the walk.
std::vector<int64_t> gemm_tile_walk_py(int64_t n_tiles, int64_t m_tiles, int64_t k_tiles, int64_t u0, int64_t u1,
                                       bool m_fastest) {
  if (n_tiles < 1 || m_tiles < 1 || k_tiles < 1 || u0 < 0 || u1 < u0 || u1 > n_tiles * m_tiles * k_tiles)
    throw std::invalid_argument("gemm_tile_walk: bad tile counts or unit range");
  hrm::TileWalk wk{(int)n_tiles, (int)m_tiles, (int)k_tiles, m_fastest ? 1 : 0, 0, 0, 0};
  std::vector<int64_t> out;
  out.reserve((size_t)(u1 - u0) * 3);
  wk.start(u0);
  for (int64_t u = u0; u < u1; ++u, wk.next()) {
    out.push_back(wk.n_tile);
    out.push_back(wk.m_tile);
    out.push_back(wk.kt);
  }
  return out;
}

std::vector<int64_t> gemm_plan_py(int64_t M, int64_t N, int64_t K, int64_t force_ctas) {
  auto p = hrm::gemm_plan((int)M, (int)N, (int)K, (int)force_ctas);
  return {p.bn, p.n_tiles, p.m_tiles, p.k_tiles, p.splits, (int64_t)p.ws_floats, p.counters, p.ku};
}

// out = x @ (w * scale)^T (+ bias): out dtype f16 or f32 (preallocated [M, >=N] row-major).
void set_in_norm(hrm::GemmArgs& a, const c10::optional<at::Tensor>& in_ssq, double inv_h, double eps) {
  if (in_ssq.has_value() && in_ssq->defined()) {
    CHECK_DTYPE((*in_ssq), at::kFloat); CHECK_CONTIG((*in_ssq));
    TORCH_CHECK(in_ssq->numel() % a.M == 0, "in_ssq must be [tiles, M]");
    a.in_ssq = in_ssq->data_ptr<float>();
    a.in_ssq_tiles = (int)(in_ssq->numel() / a.M);
    a.in_inv_h = (float)inv_h;
    a.in_eps = (float)eps;
  }
}

// Plain output [M, >= N] f16 or f32: returns the epilogue.
int fill_out(hrm::GemmArgs& a, const at::Tensor& out) {
  CHECK_CUDA(out);
  TORCH_CHECK(out.dim() == 2 && out.size(0) == a.M && out.size(1) >= a.N && out.stride(1) == 1, "bad out shape");
  int epi;
  if (out.scalar_type() == at::kHalf) epi = hrm::EPI_F16;
  else if (out.scalar_type() == at::kFloat) epi = hrm::EPI_F32;
  else TORCH_CHECK(false, "out must be f16 or f32");
  a.out = out.data_ptr();
  a.ldo = (int)out.stride(0);
  return epi;
}

void w8a16_gemm(at::Tensor x, at::Tensor w, at::Tensor scale, c10::optional<at::Tensor> bias, at::Tensor out,
                at::Tensor ws, at::Tensor counters, int64_t force_ctas, c10::optional<at::Tensor> in_ssq,
                double inv_h, double eps) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, scale, bias, ws, counters);
  set_in_norm(a, in_ssq, inv_h, eps);
  if (a.M == 0) return;
  const int epi = fill_out(a, out);
  auto p = hrm::gemm_plan(a.M, a.N, a.K, (int)force_ctas);
  check_ws(p, ws, counters);
  hrm::gemm_w8a16_launch(x.data_ptr(), (int)x.stride(0), w.data_ptr<int8_t>(), epi, a, p, cur_stream());
}

// resid += x @ (w * scale)^T  (fp32 residual stream)
// Residual epilogue fields (resid += acc; optional next-norm outputs).
void fill_resid(hrm::GemmArgs& a, const at::Tensor& resid, const c10::optional<at::Tensor>& gamma_next,
                const c10::optional<at::Tensor>& xg_out, const c10::optional<at::Tensor>& ssq_out) {
  if (xg_out.has_value() && xg_out->defined()) {
    TORCH_CHECK(gamma_next.has_value() && gamma_next->defined(), "xg_out needs gamma_next");
    CHECK_DTYPE((*xg_out), at::kHalf); CHECK_DTYPE((*gamma_next), at::kFloat);
    TORCH_CHECK(xg_out->stride(1) == 1 && gamma_next->numel() == a.N, "bad xg_out / gamma_next");
    a.xg_out = reinterpret_cast<__half*>(xg_out->data_ptr());
    a.ldxg = (int)xg_out->stride(0);
    a.gamma_next = gamma_next->data_ptr<float>();
  }
  if (ssq_out.has_value() && ssq_out->defined()) {
    CHECK_DTYPE((*ssq_out), at::kFloat);
    TORCH_CHECK(ssq_out->numel() >= (int64_t)((a.N + 127) / 128) * a.M, "ssq_out too small");
    a.ssq_out = ssq_out->data_ptr<float>();
  }
  CHECK_CUDA(resid); CHECK_DTYPE(resid, at::kFloat);
  TORCH_CHECK(resid.dim() == 2 && resid.size(0) == a.M && resid.size(1) == a.N && resid.stride(1) == 1,
              "bad resid shape");
  a.resid = resid.data_ptr<float>();
  a.ldr = (int)resid.stride(0);
}

void w8a16_gemm_residual(at::Tensor x, at::Tensor w, at::Tensor scale, at::Tensor resid, at::Tensor ws,
                         at::Tensor counters, int64_t force_ctas, c10::optional<at::Tensor> gamma_next,
                         c10::optional<at::Tensor> xg_out, c10::optional<at::Tensor> ssq_out) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, scale, c10::nullopt, ws, counters);
  if (a.M == 0) return;
  fill_resid(a, resid, gamma_next, xg_out, ssq_out);
  auto p = hrm::gemm_plan(a.M, a.N, a.K, (int)force_ctas);
  check_ws(p, ws, counters);
  hrm::gemm_w8a16_launch(x.data_ptr(), (int)x.stride(0), w.data_ptr<int8_t>(), hrm::EPI_RESID, a, p, cur_stream());
}

void fill_resid_ar(hrm::GemmArgs& a, const at::Tensor& resid, const at::Tensor& gamma_next, const at::Tensor& xg_out,
                   const at::Tensor& ssq_out, const at::Tensor& peers, int64_t rank, int64_t world,
                   int64_t off_partials, int64_t off_final, int64_t off_flags, int64_t tile_floats, int64_t max_tiles,
                   int64_t epoch_ptr, const at::Tensor& launch_ticket, int64_t off_tile_flags, int64_t off_ll,
                   int64_t ll);

// Tensor-parallel residual GEMM fused with the all-reduce over peer memory (decode, M <= 64):
//   resid = resid + sum_ranks(x_r @ W_r^T);  xg = resid * gamma_next;  ssq = per-tile sums of squares.
void w8a16_gemm_residual_ar(at::Tensor x, at::Tensor w, at::Tensor scale, at::Tensor resid, at::Tensor ws,
                            at::Tensor counters, at::Tensor gamma_next, at::Tensor xg_out, at::Tensor ssq_out,
                            at::Tensor peers, int64_t rank, int64_t world, int64_t off_partials, int64_t off_final,
                            int64_t off_flags, int64_t tile_floats, int64_t max_tiles, int64_t epoch_ptr,
                            at::Tensor launch_ticket, int64_t off_tile_flags, int64_t off_ll, int64_t ll) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, scale, c10::nullopt, ws, counters);
  if (a.M == 0) return;
  fill_resid_ar(a, resid, gamma_next, xg_out, ssq_out, peers, rank, world, off_partials, off_final, off_flags,
                tile_floats, max_tiles, epoch_ptr, launch_ticket, off_tile_flags, off_ll, ll);
  auto p = hrm::gemm_plan(a.M, a.N, a.K, 0);
  check_ws(p, ws, counters);
  hrm::gemm_w8a16_launch(x.data_ptr(), (int)x.stride(0), w.data_ptr<int8_t>(), hrm::EPI_RESID_AR, a, p,
                         cur_stream());
}

void fill_resid_ar(hrm::GemmArgs& a, const at::Tensor& resid, const at::Tensor& gamma_next, const at::Tensor& xg_out,
                   const at::Tensor& ssq_out, const at::Tensor& peers, int64_t rank, int64_t world,
                   int64_t off_partials, int64_t off_final, int64_t off_flags, int64_t tile_floats, int64_t max_tiles,
                   int64_t epoch_ptr, const at::Tensor& launch_ticket, int64_t off_tile_flags, int64_t off_ll,
                   int64_t ll) {
  CHECK_DTYPE(resid, at::kFloat); CHECK_DTYPE(gamma_next, at::kFloat); CHECK_DTYPE(xg_out, at::kHalf);
  CHECK_DTYPE(ssq_out, at::kFloat); CHECK_DTYPE(peers, at::kLong); CHECK_DTYPE(launch_ticket, at::kInt);
  TORCH_CHECK(resid.size(0) == a.M && resid.size(1) == a.N && resid.stride(1) == 1, "bad resid");
  TORCH_CHECK(peers.numel() == world && rank < world, "bad peer table");
  TORCH_CHECK(a.N % 128 == 0 && a.M <= 64, "fused all-reduce needs N % 128 == 0 and M <= 64");
  TORCH_CHECK((int64_t)a.M * 128 <= tile_floats, "symmetric tile slot too small for M");
  a.resid = resid.data_ptr<float>();
  a.ldr = (int)resid.stride(0);
  a.gamma_next = gamma_next.data_ptr<float>();
  a.xg_out = reinterpret_cast<__half*>(xg_out.data_ptr());
  a.ldxg = (int)xg_out.stride(0);
  a.ssq_out = ssq_out.data_ptr<float>();
  a.peers = reinterpret_cast<const long long*>(peers.data_ptr<int64_t>());
  a.tp_rank = (int)rank;
  a.tp_world = (int)world;
  a.off_partials = off_partials;
  a.off_final = off_final;
  a.off_flags = off_flags;
  a.off_tile_flags = off_tile_flags;
  a.off_ll = off_ll;
  a.ar_ll = ll != 0 ? 1 : 0;
  a.ar_tile_floats = (int)tile_floats;
  a.ar_max_tiles = (int)max_tiles;
  a.epoch = reinterpret_cast<int*>((uintptr_t)epoch_ptr);
  a.launch_ticket = launch_ticket.data_ptr<int>();
}

void fill_swiglu(hrm::GemmArgs& a, const at::Tensor& out) {
  CHECK_CUDA(out); CHECK_DTYPE(out, at::kHalf);
  TORCH_CHECK(out.dim() == 2 && out.size(0) == a.M && out.size(1) == a.N / 2 && out.stride(1) == 1, "bad out");
  a.out = out.data_ptr();
  a.ldo = (int)out.stride(0);
}

// out [M, N/2] f16 = silu(gate) * up, where w rows are interleaved per 128-row tile: 64 gate rows then the 64
// matching up rows.
void w8a16_gemm_swiglu(at::Tensor x, at::Tensor w, at::Tensor scale, at::Tensor out, at::Tensor ws,
                       at::Tensor counters, int64_t force_ctas, c10::optional<at::Tensor> in_ssq, double inv_h,
                       double eps) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, scale, c10::nullopt, ws, counters);
  set_in_norm(a, in_ssq, inv_h, eps);
  if (a.M == 0) return;
  fill_swiglu(a, out);
  auto p = hrm::gemm_plan(a.M, a.N, a.K, (int)force_ctas);
  check_ws(p, ws, counters);
  hrm::gemm_w8a16_launch(x.data_ptr(), (int)x.stride(0), w.data_ptr<int8_t>(), hrm::EPI_SWIGLU, a, p, cur_stream());
}

// Fused QKV projection + bias + RoPE + paged-KV append.  w rows: [q (q_rows) | k (kv_rows) | v (kv_rows)].
void fill_qkv(hrm::GemmArgs& a, int64_t q_rows, int64_t kv_rows, int64_t head_dim, const at::Tensor& positions,
              const at::Tensor& slots, const at::Tensor& cos_t, const at::Tensor& sin_t, const at::Tensor& q_out,
              const at::Tensor& k_cache, const at::Tensor& v_cache);

void w8a16_gemm_qkv(at::Tensor x, at::Tensor w, at::Tensor scale, c10::optional<at::Tensor> bias, int64_t q_rows,
                    int64_t kv_rows, int64_t head_dim, at::Tensor positions, at::Tensor slots, at::Tensor cos_t,
                    at::Tensor sin_t, at::Tensor q_out, at::Tensor k_cache, at::Tensor v_cache, at::Tensor ws,
                    at::Tensor counters, int64_t force_ctas, c10::optional<at::Tensor> in_ssq, double inv_h,
                    double eps) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = base_args(x, w, scale, bias, ws, counters);
  set_in_norm(a, in_ssq, inv_h, eps);
  if (a.M == 0) return;
  fill_qkv(a, q_rows, kv_rows, head_dim, positions, slots, cos_t, sin_t, q_out, k_cache, v_cache);
  auto p = hrm::gemm_plan(a.M, a.N, a.K, (int)force_ctas);
  check_ws(p, ws, counters);
  hrm::gemm_w8a16_launch(x.data_ptr(), (int)x.stride(0), w.data_ptr<int8_t>(), hrm::EPI_QKV, a, p, cur_stream());
}

void fill_qkv(hrm::GemmArgs& a, int64_t q_rows, int64_t kv_rows, int64_t head_dim, const at::Tensor& positions,
              const at::Tensor& slots, const at::Tensor& cos_t, const at::Tensor& sin_t, const at::Tensor& q_out,
              const at::Tensor& k_cache, const at::Tensor& v_cache) {
  TORCH_CHECK(a.N == q_rows + 2 * kv_rows, "w rows must be q_rows + 2*kv_rows");
  CHECK_DTYPE(positions, at::kInt); CHECK_DTYPE(slots, at::kInt);
  CHECK_DTYPE(cos_t, at::kFloat); CHECK_DTYPE(sin_t, at::kFloat);
  CHECK_DTYPE(q_out, at::kBFloat16); CHECK_DTYPE(k_cache, at::kBFloat16); CHECK_DTYPE(v_cache, at::kBFloat16);
  CHECK_CONTIG(q_out); CHECK_CONTIG(k_cache); CHECK_CONTIG(v_cache); CHECK_CONTIG(cos_t); CHECK_CONTIG(sin_t);
  TORCH_CHECK(positions.numel() >= a.M && slots.numel() >= a.M, "positions/slots too short");
  TORCH_CHECK(q_out.numel() >= (int64_t)a.M * q_rows, "q_out too small");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == head_dim, "k_cache must be [blocks, Hk, bs, D]");
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes(), "k/v cache shape mismatch");
  TORCH_CHECK(cos_t.size(1) == head_dim / 2, "rope table width must be head_dim/2");
  a.q_rows = (int)q_rows;
  a.kv_rows = (int)kv_rows;
  a.head_dim = (int)head_dim;
  a.kv_heads = (int)k_cache.size(1);
  a.block_size = (int)k_cache.size(2);
  TORCH_CHECK(a.kv_heads * head_dim == kv_rows, "kv_rows must equal cache kv_heads * head_dim");
  a.positions = positions.data_ptr<int>();
  a.slots = slots.data_ptr<int>();
  a.cos_t = cos_t.data_ptr<float>();
  a.sin_t = sin_t.data_ptr<float>();
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  a.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
}

// Multi-phase decode chain in one cooperative launch.  `phases` is a list of tuples, phase p + 1 reading phase p's
// outputs:
//   ("f16",    x, w, scale, out, in_ssq | None, inv_h, eps)
//   ("resid",  x, w, scale, resid, gamma_next | None, xg_out | None, ssq_out | None)
//   ("swiglu", x, w, scale, out, in_ssq | None, inv_h, eps)
//   ("qkv",    x, w, scale, bias | None, q_rows, kv_rows, head_dim, positions, slots, cos, sin, q_out, k_cache,
//              v_cache, in_ssq | None, inv_h, eps)
// w: pre-tiled int8 weights.  ws / counters: split-K scratch covering every phase; bar: int32 [5] zero at rest.
static c10::optional<at::Tensor> opt_tensor(const py::handle& h) {
  if (h.is_none()) return c10::nullopt;
  return h.cast<at::Tensor>();
}

void w8a16_chain(py::list phases, at::Tensor ws, at::Tensor counters, at::Tensor bar) {
  const int nph = (int)py::len(phases);
  TORCH_CHECK(nph >= 1 && nph <= hrm::kMaxChainPhases, "chain: 1..4 phases");
  CHECK_CUDA(bar); CHECK_DTYPE(bar, at::kInt);
  TORCH_CHECK(bar.numel() >= hrm::kMaxChainPhases + 1, "chain: bar needs 5 int32");
  std::vector<hrm::ChainPhaseDesc> d(nph);
  c10::optional<c10::cuda::CUDAGuard> guard;
  const int G = hrm::gemm_sm_count();
  for (int p = 0; p < nph; ++p) {
    py::tuple t = phases[p].cast<py::tuple>();
    const std::string kind = t[0].cast<std::string>();
    at::Tensor x = t[1].cast<at::Tensor>(), w = t[2].cast<at::Tensor>(), scale = t[3].cast<at::Tensor>();
    if (!guard) guard.emplace(x.device());
    TORCH_CHECK(w.dim() == 3, "chain: pre-tiled weights required");
    hrm::GemmArgs a;
    if (kind == "f16") {
      a = base_args(x, w, scale, c10::nullopt, ws, counters);
      set_in_norm(a, opt_tensor(t[5]), t[6].cast<double>(), t[7].cast<double>());
      d[p].epi = fill_out(a, t[4].cast<at::Tensor>());
      TORCH_CHECK(d[p].epi == hrm::EPI_F16, "chain: f16 output only");
    } else if (kind == "resid") {
      a = base_args(x, w, scale, c10::nullopt, ws, counters);
      fill_resid(a, t[4].cast<at::Tensor>(), opt_tensor(t[5]), opt_tensor(t[6]), opt_tensor(t[7]));
      d[p].epi = hrm::EPI_RESID;
    } else if (kind == "resid_ar") {
      // ("resid_ar", x, w, scale, resid, gamma_next, xg_out, ssq_out, peers, rank, world, off_partials, off_final,
      //  off_flags, tile_floats, max_tiles, epoch_ptr, launch_ticket)
      a = base_args(x, w, scale, c10::nullopt, ws, counters);
      fill_resid_ar(a, t[4].cast<at::Tensor>(), t[5].cast<at::Tensor>(), t[6].cast<at::Tensor>(),
                    t[7].cast<at::Tensor>(), t[8].cast<at::Tensor>(), t[9].cast<int64_t>(), t[10].cast<int64_t>(),
                    t[11].cast<int64_t>(), t[12].cast<int64_t>(), t[13].cast<int64_t>(), t[14].cast<int64_t>(),
                    t[15].cast<int64_t>(), t[16].cast<int64_t>(), t[17].cast<at::Tensor>(), 0, 0, 0);
      d[p].epi = hrm::EPI_RESID_AR;
    } else if (kind == "swiglu") {
      a = base_args(x, w, scale, c10::nullopt, ws, counters);
      set_in_norm(a, opt_tensor(t[5]), t[6].cast<double>(), t[7].cast<double>());
      fill_swiglu(a, t[4].cast<at::Tensor>());
      d[p].epi = hrm::EPI_SWIGLU;
    } else if (kind == "qkv") {
      a = base_args(x, w, scale, opt_tensor(t[4]), ws, counters);
      set_in_norm(a, opt_tensor(t[15]), t[16].cast<double>(), t[17].cast<double>());
      fill_qkv(a, t[5].cast<int64_t>(), t[6].cast<int64_t>(), t[7].cast<int64_t>(), t[8].cast<at::Tensor>(),
               t[9].cast<at::Tensor>(), t[10].cast<at::Tensor>(), t[11].cast<at::Tensor>(), t[12].cast<at::Tensor>(),
               t[13].cast<at::Tensor>(), t[14].cast<at::Tensor>());
      d[p].epi = hrm::EPI_QKV;
    } else {
      TORCH_CHECK(false, "chain: unknown phase kind ", kind);
    }
    TORCH_CHECK(a.M > 0 && a.M <= 32, "chain: 1 <= M <= 32");
    check_ws(hrm::gemm_chain_phase_plan(a.M, a.N, a.K, G), ws, counters);
    d[p].x = x.data_ptr();
    d[p].ldx = (int)x.stride(0);
    d[p].a = a;
  }
  hrm::gemm_chain_launch(d.data(), nph, bar.data_ptr<int>(), cur_stream());
}

std::vector<int64_t> chain_phase_plan_py(int64_t M, int64_t N, int64_t K) {
  auto p = hrm::gemm_chain_phase_plan((int)M, (int)N, (int)K, hrm::gemm_sm_count());
  return {p.bn, (int64_t)p.ws_floats, p.counters};
}

void rmsnorm(at::Tensor x, c10::optional<at::Tensor> delta, at::Tensor w, double eps, at::Tensor out) {
  c10::cuda::CUDAGuard g(x.device());
  CHECK_CUDA(x); CHECK_DTYPE(x, at::kFloat); CHECK_CONTIG(x);
  CHECK_DTYPE(w, at::kFloat); CHECK_DTYPE(out, at::kHalf); CHECK_CONTIG(out);
  const int H = (int)x.size(-1);
  const int M = (int)(x.numel() / H);
  TORCH_CHECK(H % 4 == 0, "hidden must be a multiple of 4");
  TORCH_CHECK(out.numel() == x.numel() && w.numel() == H, "shape mismatch");
  const float* d = nullptr;
  if (delta.has_value() && delta->defined()) {
    CHECK_DTYPE((*delta), at::kFloat); CHECK_CONTIG((*delta));
    TORCH_CHECK(delta->numel() == x.numel(), "delta shape mismatch");
    d = delta->data_ptr<float>();
  }
  hrm::rmsnorm_launch(x.data_ptr<float>(), d, w.data_ptr<float>(), reinterpret_cast<__half*>(out.data_ptr()), M, H,
                      (float)eps, cur_stream());
}

void norm_prep(at::Tensor x, c10::optional<at::Tensor> delta, at::Tensor gamma, at::Tensor xg, at::Tensor ssq) {
  c10::cuda::CUDAGuard g(x.device());
  CHECK_DTYPE(x, at::kFloat); CHECK_CONTIG(x); CHECK_DTYPE(gamma, at::kFloat); CHECK_DTYPE(xg, at::kHalf);
  CHECK_CONTIG(xg); CHECK_DTYPE(ssq, at::kFloat); CHECK_CONTIG(ssq);
  const int H = (int)x.size(-1);
  const int M = (int)(x.numel() / H);
  TORCH_CHECK(H % 128 == 0, "hidden must be a multiple of 128");
  TORCH_CHECK(xg.numel() == x.numel() && ssq.numel() >= (int64_t)(H / 128) * M, "shape mismatch");
  const float* d = nullptr;
  if (delta.has_value() && delta->defined()) {
    CHECK_DTYPE((*delta), at::kFloat); CHECK_CONTIG((*delta));
    d = delta->data_ptr<float>();
  }
  hrm::norm_prep_launch(x.data_ptr<float>(), d, gamma.data_ptr<float>(), reinterpret_cast<__half*>(xg.data_ptr()),
                        ssq.data_ptr<float>(), M, H, cur_stream());
}

void embed_q8(at::Tensor ids, at::Tensor q, at::Tensor scale, int64_t vocab_start, at::Tensor out) {
  c10::cuda::CUDAGuard g(ids.device());
  CHECK_DTYPE(ids, at::kLong); CHECK_DTYPE(q, at::kChar); CHECK_DTYPE(scale, at::kFloat); CHECK_DTYPE(out, at::kFloat);
  CHECK_CONTIG(ids); CHECK_CONTIG(q); CHECK_CONTIG(out);
  const int H = (int)q.size(1);
  TORCH_CHECK(H % 4 == 0 && out.numel() == ids.numel() * H, "shape mismatch");
  hrm::embed_q8_launch(ids.data_ptr<int64_t>(), q.data_ptr<int8_t>(), scale.data_ptr<float>(), out.data_ptr<float>(),
                       (int)ids.numel(), H, (int)vocab_start, (int)q.size(0), cur_stream());
}

int64_t decode_attention(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor block_tables,
                         at::Tensor context_lens, at::Tensor out, at::Tensor ws, int64_t splits,
                         int64_t keys_per_split, double scale, c10::optional<at::Tensor> status, bool allow_tc,
                         bool kv_prefetch, c10::optional<at::Tensor> tickets) {
  c10::cuda::CUDAGuard g(q.device());
  CHECK_DTYPE(q, at::kBFloat16); CHECK_DTYPE(k_cache, at::kBFloat16); CHECK_DTYPE(v_cache, at::kBFloat16);
  CHECK_DTYPE(block_tables, at::kInt); CHECK_DTYPE(context_lens, at::kInt); CHECK_DTYPE(out, at::kHalf);
  CHECK_CONTIG(q); CHECK_CONTIG(k_cache); CHECK_CONTIG(v_cache); CHECK_CONTIG(block_tables); CHECK_CONTIG(out);
  TORCH_CHECK(q.dim() == 3, "q must be [B, Hq, D]");
  hrm::DecodeAttnArgs a{};
  a.B = (int)q.size(0); a.Hq = (int)q.size(1); a.D = (int)q.size(2);
  a.Hk = (int)k_cache.size(1); a.block_size = (int)k_cache.size(2);
  a.max_blocks = (int)block_tables.size(1);
  a.splits = (int)splits; a.keys_per_split = (int)keys_per_split;
  a.scale = (float)scale;
  a.kv_prefetch = kv_prefetch ? 1 : 0;
  TORCH_CHECK(a.Hq % a.Hk == 0, "Hq must be a multiple of Hk");
  TORCH_CHECK(out.numel() == q.numel(), "out shape mismatch");
  if (a.splits > 1) {
    CHECK_DTYPE(ws, at::kFloat);
    TORCH_CHECK((size_t)ws.numel() >= hrm::decode_attn_ws_floats(a.B, a.Hq, a.D, a.splits), "attention ws too small");
    a.ws = ws.data_ptr<float>();
  }
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.context_lens = context_lens.data_ptr<int>();
  a.out = reinterpret_cast<__half*>(out.data_ptr());
  if (a.B == 0) return 0;
  int* st = nullptr;
  if (status.has_value() && status->defined()) { CHECK_DTYPE((*status), at::kInt); st = status->data_ptr<int>(); }
  if (allow_tc && hrm::decode_attn_tc_supported(a)) {
    if (a.splits > 1 && tickets.has_value() && tickets->defined() &&
        (a.Hq / a.Hk) * a.splits <= hrm::decode_attn_tc_merge_max()) {
      CHECK_DTYPE((*tickets), at::kInt);
      TORCH_CHECK(tickets->numel() >= (int64_t)a.B * a.Hk, "attention tickets: need B * Hk int32");
      a.tickets = tickets->data_ptr<int>();
    }
    hrm::decode_attn_tc_launch(a, (int)k_cache.size(0), st, cur_stream());
    return (a.splits > 1 && a.tickets == nullptr) ? 2 : 1;
  }
  hrm::decode_attn_launch(a, cur_stream());
  return a.splits > 1 ? 2 : 1;
}

void prefill_attention(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor block_tables,
                       at::Tensor cu_q, at::Tensor q_start, at::Tensor context_lens, at::Tensor out, int64_t max_q,
                       double scale, bool allow_tc) {
  c10::cuda::CUDAGuard g(q.device());
  CHECK_DTYPE(q, at::kBFloat16); CHECK_DTYPE(k_cache, at::kBFloat16); CHECK_DTYPE(v_cache, at::kBFloat16);
  CHECK_DTYPE(block_tables, at::kInt); CHECK_DTYPE(cu_q, at::kInt); CHECK_DTYPE(q_start, at::kInt);
  CHECK_DTYPE(context_lens, at::kInt); CHECK_DTYPE(out, at::kHalf);
  CHECK_CONTIG(q); CHECK_CONTIG(k_cache); CHECK_CONTIG(v_cache); CHECK_CONTIG(block_tables); CHECK_CONTIG(out);
  TORCH_CHECK(q.dim() == 3, "q must be [Tq, Hq, D]");
  hrm::PrefillAttnArgs a{};
  a.Hq = (int)q.size(1); a.D = (int)q.size(2);
  a.Hk = (int)k_cache.size(1); a.block_size = (int)k_cache.size(2);
  a.S = (int)q_start.numel(); a.max_blocks = (int)block_tables.size(1); a.max_q = (int)max_q;
  a.scale = (float)scale;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.cu_q = cu_q.data_ptr<int>();
  a.q_start = q_start.data_ptr<int>();
  a.context_lens = context_lens.data_ptr<int>();
  a.out = reinterpret_cast<__half*>(out.data_ptr());
  if (allow_tc && hrm::prefill_attn_tc_supported(a))
    hrm::prefill_attn_tc_launch(a, (int)k_cache.size(0), (int)q.size(0), nullptr, cur_stream());
  else
    hrm::prefill_attn_launch(a, cur_stream());
}

void argmax_rows(at::Tensor logits, int64_t vocab_start, c10::optional<at::Tensor> keys, at::Tensor tokens,
                 c10::optional<at::Tensor> scratch) {
  c10::cuda::CUDAGuard g(logits.device());
  CHECK_DTYPE(logits, at::kFloat); CHECK_DTYPE(tokens, at::kLong);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be [M, V] row-major");
  unsigned long long* kp = nullptr;
  if (keys.has_value() && keys->defined()) {
    CHECK_DTYPE((*keys), at::kLong);
    kp = reinterpret_cast<unsigned long long*>(keys->data_ptr<int64_t>());
  }
  unsigned long long* sp = nullptr;
  if (scratch.has_value() && scratch->defined()) {
    CHECK_DTYPE((*scratch), at::kLong);
    TORCH_CHECK(scratch->numel() >= 2 * hrm::kArgmaxMaxRows, "argmax scratch: int64[2 * 4096]");
    sp = reinterpret_cast<unsigned long long*>(scratch->data_ptr<int64_t>());
  }
  hrm::argmax_launch(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1), (int)logits.stride(0),
                     (int)vocab_start, kp, tokens.data_ptr<int64_t>(), sp, hrm::gemm_sm_count(), cur_stream());
}

void argmax_rows_xchg(at::Tensor logits, int64_t vocab_start, at::Tensor tokens, c10::optional<at::Tensor> scratch,
                      at::Tensor peers, int64_t rank, int64_t world, int64_t max_rows, int64_t off_keys,
                      int64_t off_flags, int64_t epoch_ptr, int64_t row_ticket_ptr) {
  c10::cuda::CUDAGuard g(logits.device());
  CHECK_DTYPE(logits, at::kFloat); CHECK_DTYPE(tokens, at::kLong); CHECK_DTYPE(peers, at::kLong);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be [M, V] row-major");
  TORCH_CHECK(peers.numel() == world && rank >= 0 && rank < world, "bad peer table");
  unsigned long long* sp = nullptr;
  if (scratch.has_value() && scratch->defined()) {
    CHECK_DTYPE((*scratch), at::kLong);
    TORCH_CHECK(scratch->numel() >= 2 * hrm::kArgmaxMaxRows, "argmax scratch: int64[2 * 4096]");
    sp = reinterpret_cast<unsigned long long*>(scratch->data_ptr<int64_t>());
  }
  hrm::ArgmaxXchg x{};
  x.peers = reinterpret_cast<const long long*>(peers.data_ptr<int64_t>());
  x.rank = (int)rank;
  x.world = (int)world;
  x.max_rows = (int)max_rows;
  x.off_keys = off_keys;
  x.off_flags = off_flags;
  x.epoch = reinterpret_cast<int*>((uintptr_t)epoch_ptr);
  x.row_ticket = reinterpret_cast<int*>((uintptr_t)row_ticket_ptr);
  x.status = hrm::status_word();
  hrm::argmax_xchg_launch(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1), (int)logits.stride(0),
                          (int)vocab_start, nullptr, tokens.data_ptr<int64_t>(), sp, hrm::gemm_sm_count(), x,
                          cur_stream());
}

// Sampled pick on the argmax path (temperature / top-k, Gumbel-max); with ``peers`` defined the rows' keys are
// exchanged over peer memory as in argmax_rows_xchg.
void argmax_rows_sample(at::Tensor logits, int64_t vocab_start, c10::optional<at::Tensor> keys, at::Tensor tokens,
                        c10::optional<at::Tensor> scratch, at::Tensor inv_temp, c10::optional<at::Tensor> thresh,
                        at::Tensor seed, at::Tensor pos, c10::optional<at::Tensor> peers, int64_t rank, int64_t world,
                        int64_t max_rows, int64_t off_keys, int64_t off_flags, int64_t epoch_ptr,
                        int64_t row_ticket_ptr) {
  c10::cuda::CUDAGuard g(logits.device());
  CHECK_DTYPE(logits, at::kFloat); CHECK_DTYPE(tokens, at::kLong);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be [M, V] row-major");
  const int64_t M = logits.size(0);
  CHECK_DTYPE(inv_temp, at::kFloat); CHECK_DTYPE(seed, at::kLong); CHECK_DTYPE(pos, at::kInt);
  for (const at::Tensor* t : {&inv_temp, &seed, &pos, &tokens})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->numel() >= M, "per-row sampling arrays: >= M entries");
  hrm::SampleArgs sa{};
  sa.inv_temp = inv_temp.data_ptr<float>();
  sa.seed = reinterpret_cast<const unsigned long long*>(seed.data_ptr<int64_t>());
  sa.pos = pos.data_ptr<int>();
  if (thresh.has_value() && thresh->defined()) {
    CHECK_DTYPE((*thresh), at::kFloat);
    TORCH_CHECK(thresh->is_contiguous() && thresh->numel() >= M, "thresh: f32 [M]");
    sa.thresh = thresh->data_ptr<float>();
  }
  unsigned long long* kp = nullptr;
  if (keys.has_value() && keys->defined()) {
    CHECK_DTYPE((*keys), at::kLong);
    kp = reinterpret_cast<unsigned long long*>(keys->data_ptr<int64_t>());
  }
  unsigned long long* sp = nullptr;
  if (scratch.has_value() && scratch->defined()) {
    CHECK_DTYPE((*scratch), at::kLong);
    TORCH_CHECK(scratch->numel() >= 2 * hrm::kArgmaxMaxRows, "argmax scratch: int64[2 * 4096]");
    sp = reinterpret_cast<unsigned long long*>(scratch->data_ptr<int64_t>());
  }
  hrm::ArgmaxXchg x{};
  const bool xchg = peers.has_value() && peers->defined();
  if (xchg) {
    CHECK_DTYPE((*peers), at::kLong);
    TORCH_CHECK(peers->numel() == world && rank >= 0 && rank < world, "bad peer table");
    x.peers = reinterpret_cast<const long long*>(peers->data_ptr<int64_t>());
    x.rank = (int)rank;
    x.world = (int)world;
    x.max_rows = (int)max_rows;
    x.off_keys = off_keys;
    x.off_flags = off_flags;
    x.epoch = reinterpret_cast<int*>((uintptr_t)epoch_ptr);
    x.row_ticket = reinterpret_cast<int*>((uintptr_t)row_ticket_ptr);
    x.status = hrm::status_word();
  }
  hrm::argmax_sample_launch(logits.data_ptr<float>(), (int)M, (int)logits.size(1), (int)logits.stride(0),
                            (int)vocab_start, kp, tokens.data_ptr<int64_t>(), sp, hrm::gemm_sm_count(), sa,
                            xchg ? &x : nullptr, cur_stream());
}

// Top-k selection helpers of the sampled pick: k-th largest per row, and each row's top-k candidate values.
void kth_largest_rows(at::Tensor x, at::Tensor k, at::Tensor out, at::Tensor state) {
  c10::cuda::CUDAGuard g(x.device());
  CHECK_DTYPE(x, at::kFloat); CHECK_DTYPE(k, at::kInt); CHECK_DTYPE(out, at::kFloat); CHECK_DTYPE(state, at::kInt);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [R, n] row-major");
  TORCH_CHECK(k.is_contiguous() && out.is_contiguous() && k.numel() >= x.size(0) && out.numel() >= x.size(0),
              "k int32 [R], out f32 [R]");
  TORCH_CHECK(state.is_contiguous() && state.numel() >= hrm::kth_largest_state_words((int)x.size(0)),
              "state: int32 [kth_largest_state_words(R)]");
  hrm::kth_largest_launch(x.data_ptr<float>(), (int)x.size(0), (int)x.size(1), (int)x.stride(0), k.data_ptr<int>(),
                          out.data_ptr<float>(), reinterpret_cast<uint32_t*>(state.data_ptr<int>()),
                          hrm::gemm_sm_count(), cur_stream());
}

void topk_candidates_rows(at::Tensor x, at::Tensor thresh, at::Tensor k, at::Tensor cand) {
  c10::cuda::CUDAGuard g(x.device());
  CHECK_DTYPE(x, at::kFloat); CHECK_DTYPE(thresh, at::kFloat);
  CHECK_DTYPE(k, at::kInt); CHECK_DTYPE(cand, at::kFloat);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [R, n] row-major");
  TORCH_CHECK(cand.dim() == 2 && cand.is_contiguous() && cand.size(0) == x.size(0), "cand: f32 [R, kmax] contiguous");
  TORCH_CHECK(thresh.is_contiguous() && k.is_contiguous() && thresh.numel() >= x.size(0) && k.numel() >= x.size(0),
              "thresh f32 [R], k int32 [R]");
  hrm::topk_candidates_launch(x.data_ptr<float>(), (int)x.size(0), (int)x.size(1), (int)x.stride(0),
                              thresh.data_ptr<float>(), k.data_ptr<int>(), (int)cand.size(1), cand.data_ptr<float>(),
                              cur_stream());
}

// C [M, N] fp32 = A [M, K] . B [N, K]^T on the tensor cores (A, B bf16 or f16, same type, unit inner stride).
void gemm_nt(at::Tensor A, at::Tensor B, at::Tensor C) {
  c10::cuda::CUDAGuard g(A.device());
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm_nt: CUDA tensors");
  TORCH_CHECK(A.scalar_type() == B.scalar_type() &&
              (A.scalar_type() == at::kBFloat16 || A.scalar_type() == at::kHalf), "gemm_nt: A, B both bf16 or f16");
  CHECK_DTYPE(C, at::kFloat);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm_nt: 2-D operands");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm_nt: unit inner stride");
  TORCH_CHECK(A.size(1) == B.size(1), "gemm_nt: K mismatch");
  TORCH_CHECK(C.size(0) == A.size(0) && C.size(1) == B.size(0), "gemm_nt: C must be [M, N]");
  hrm::gemm_nt_launch(A.data_ptr(), (int)A.stride(0), B.data_ptr(), (int)B.stride(0), C.data_ptr<float>(),
                      (int)C.stride(0), (int)A.size(0), (int)B.size(0), (int)A.size(1),
                      A.scalar_type() == at::kBFloat16, nullptr, cur_stream());
}

// Trainer causal attention: every operand contiguous fp32 [B, T, H, D] (D 16 or 32) on one device, lse [B, H, T].
static void check_flash_train(std::initializer_list<const at::Tensor*> ts, const at::Tensor& ref,
                              const at::Tensor& lse) {
  TORCH_CHECK(ref.dim() == 4 && (ref.size(3) == 16 || ref.size(3) == 32), "flash_train: [B, T, H, D] with D 16 or 32");
  for (const at::Tensor* t : ts) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->sizes() == ref.sizes() &&
                    t->device() == ref.device(), "flash_train: contiguous f32 CUDA tensors of one shape and device");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0, "flash_train: 16-byte aligned operands");
  }
  TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.device() == ref.device() &&
                  lse.dim() == 3 && lse.size(0) == ref.size(0) && lse.size(1) == ref.size(2) && lse.size(2) == ref.size(1),
              "flash_train: lse contiguous f32 [B, H, T] on the same device");
}

void flash_train_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, int64_t rpt) {
  c10::cuda::CUDAGuard g(q.device());
  check_flash_train({&q, &k, &v, &o}, q, lse);
  hrm::flash_train_fwd_launch(q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), o.data_ptr<float>(),
                              lse.data_ptr<float>(), (int)q.size(0), (int)q.size(1), (int)q.size(2), (int)q.size(3),
                              (int)rpt, cur_stream());
}

void flash_train_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, at::Tensor dout,
                     at::Tensor dq, at::Tensor dk, at::Tensor dv, int64_t rpt) {
  c10::cuda::CUDAGuard g(q.device());
  check_flash_train({&q, &k, &v, &o, &dout, &dq, &dk, &dv}, q, lse);
  hrm::flash_train_bwd_launch(q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), o.data_ptr<float>(),
                              lse.data_ptr<float>(), dout.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr<float>(),
                              dv.data_ptr<float>(), (int)q.size(0), (int)q.size(1), (int)q.size(2), (int)q.size(3),
                              (int)rpt, cur_stream());
}

void decode_prepare_bs(at::Tensor positions, at::Tensor tables, int64_t block_size, c10::optional<at::Tensor> active,
                       at::Tensor slots, at::Tensor context_lens) {
  c10::cuda::CUDAGuard g(positions.device());
  CHECK_DTYPE(positions, at::kInt); CHECK_DTYPE(tables, at::kInt); CHECK_DTYPE(slots, at::kInt);
  CHECK_DTYPE(context_lens, at::kInt); CHECK_CONTIG(tables);
  const int* ap = nullptr;
  if (active.has_value() && active->defined()) { CHECK_DTYPE((*active), at::kInt); ap = active->data_ptr<int>(); }
  hrm::decode_prepare_launch(positions.data_ptr<int>(), tables.data_ptr<int>(), (int)tables.size(1),
                             (int)block_size, ap, slots.data_ptr<int>(), context_lens.data_ptr<int>(),
                             (int)positions.numel(), cur_stream());
}

void decode_advance(at::Tensor tokens, at::Tensor ids, at::Tensor positions, c10::optional<at::Tensor> active) {
  c10::cuda::CUDAGuard g(tokens.device());
  CHECK_DTYPE(tokens, at::kLong); CHECK_DTYPE(ids, at::kLong); CHECK_DTYPE(positions, at::kInt);
  const int* ap = nullptr;
  if (active.has_value() && active->defined()) { CHECK_DTYPE((*active), at::kInt); ap = active->data_ptr<int>(); }
  hrm::decode_advance_launch(tokens.data_ptr<int64_t>(), ids.data_ptr<int64_t>(), positions.data_ptr<int>(), ap,
                             (int)positions.numel(), cur_stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of hrm_flashrenderer_b200";
  m.def("gemm_plan", &gemm_plan_py, "stream-K plan: (bn, n_tiles, m_tiles, units per tile, splits, ws_floats, counters, k-tiles per unit)");
  m.def("w8a16_gemm", &w8a16_gemm, py::arg("x"), py::arg("w"), py::arg("scale"), py::arg("bias"), py::arg("out"),
        py::arg("ws"), py::arg("counters"), py::arg("force_ctas") = 0, py::arg("in_ssq") = py::none(),
        py::arg("inv_h") = 0.0, py::arg("eps") = 0.0);
  m.def("w8a16_gemm_residual", &w8a16_gemm_residual, py::arg("x"), py::arg("w"), py::arg("scale"), py::arg("resid"),
        py::arg("ws"), py::arg("counters"), py::arg("force_ctas") = 0, py::arg("gamma_next") = py::none(),
        py::arg("xg_out") = py::none(), py::arg("ssq_out") = py::none());
  m.def("w8a16_gemm_residual_ar", &w8a16_gemm_residual_ar);
  m.def("w8a16_gemm_swiglu", &w8a16_gemm_swiglu, py::arg("x"), py::arg("w"), py::arg("scale"), py::arg("out"),
        py::arg("ws"), py::arg("counters"), py::arg("force_ctas") = 0, py::arg("in_ssq") = py::none(),
        py::arg("inv_h") = 0.0, py::arg("eps") = 0.0);
  m.def("w8a16_gemm_qkv", &w8a16_gemm_qkv, py::arg("x"), py::arg("w"), py::arg("scale"), py::arg("bias"),
        py::arg("q_rows"), py::arg("kv_rows"), py::arg("head_dim"), py::arg("positions"), py::arg("slots"),
        py::arg("cos_t"), py::arg("sin_t"), py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"), py::arg("ws"),
        py::arg("counters"), py::arg("force_ctas") = 0, py::arg("in_ssq") = py::none(), py::arg("inv_h") = 0.0,
        py::arg("eps") = 0.0);
  m.def("rmsnorm", &rmsnorm);
  m.def("embed_q8", &embed_q8);
  m.def("norm_prep", &norm_prep);
  m.def("decode_attention", &decode_attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("context_lens"), py::arg("out"), py::arg("ws"), py::arg("splits"),
        py::arg("keys_per_split"), py::arg("scale"), py::arg("status") = py::none(), py::arg("allow_tc") = true,
        py::arg("kv_prefetch") = false, py::arg("tickets") = py::none());
  m.def("decode_attn_ws_floats", [](int64_t B, int64_t Hq, int64_t D, int64_t s) {
    return (int64_t)hrm::decode_attn_ws_floats((int)B, (int)Hq, (int)D, (int)s);
  });
  m.def("prefill_attention", &prefill_attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("cu_q"), py::arg("q_start"), py::arg("context_lens"), py::arg("out"),
        py::arg("max_q"), py::arg("scale"), py::arg("allow_tc") = true);
  m.def("argmax_rows", &argmax_rows, py::arg("logits"), py::arg("vocab_start"), py::arg("keys"), py::arg("tokens"),
        py::arg("scratch") = py::none());
  m.def("decode_prepare", &decode_prepare_bs);
  m.def("decode_advance", &decode_advance);
  // per CTA and segment of the even stream-K split: (cta, tile, nseg, segidx), for the host-side test
  m.def("stream_k_segments", [](int64_t tiles, int64_t k_tiles, int64_t G) {
    std::vector<int64_t> out;
    const long long U = tiles * k_tiles;
    for (long long c = 0; c < G; ++c) {
      const long long u0 = c * U / G, u1 = (c + 1) * U / G;
      for (long long u = u0; u < u1;) {
        const long long tile = u / k_tiles, f = tile * k_tiles, end = std::min(f + k_tiles, u1);
        int nseg = 0, segidx = 0;
        hrm::tile_segments(f, (int)k_tiles, u, U, G, nseg, segidx);
        out.insert(out.end(), {c, tile, nseg, segidx});
        u = end;
      }
    }
    return out;
  });
  m.def("sm_count", []() { return hrm::gemm_sm_count(); });
  m.def("argmax_rows_xchg", &argmax_rows_xchg);
  m.def("argmax_rows_sample", &argmax_rows_sample, "temperature / top-k sampled pick on the argmax path");
  m.def("kth_largest_rows", &kth_largest_rows, "k-th largest value of every row (radix select)");
  m.def("kth_largest_state_words", [](int64_t rows) { return (int64_t)hrm::kth_largest_state_words((int)rows); });
  m.def("topk_candidates_rows", &topk_candidates_rows, "each row's top-k candidate values");
  m.def("gemm_nt", &gemm_nt);
  m.def("flash_train_fwd", &flash_train_fwd, "trainer causal attention forward (o, lse)", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("rpt") = 2);
  m.def("flash_train_bwd", &flash_train_bwd, "trainer causal attention backward (dq, dk, dv)", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("dout"), py::arg("dq"), py::arg("dk"),
        py::arg("dv"), py::arg("rpt") = 2);
  m.def("grad_clip_factor", [](at::Tensor g, double clip, at::Tensor partial, at::Tensor scalars) {
    c10::cuda::CUDAGuard gd(g.device());
    TORCH_CHECK(g.is_cuda() && g.scalar_type() == at::kFloat && g.is_contiguous(), "g: contiguous f32 CUDA");
    TORCH_CHECK(partial.numel() >= 1024 && scalars.numel() >= 2, "partial[1024], scalars[2]");
    hrm::grad_clip_factor_launch(g.data_ptr<float>(), g.numel(), (float)clip, partial.data_ptr<float>(),
                                 scalars.data_ptr<float>(), cur_stream());
  });
  m.def("adamw_flat", [](at::Tensor w, at::Tensor m_, at::Tensor v, at::Tensor g, double lr, double wd, double b1,
                         double b2, double eps, at::Tensor step, at::Tensor scalars) {
    c10::cuda::CUDAGuard gd(w.device());
    for (auto* t : {&w, &m_, &v, &g})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == w.numel(),
                  "w, m, v, g: contiguous f32 CUDA of one size");
    TORCH_CHECK(step.scalar_type() == at::kInt && scalars.scalar_type() == at::kFloat, "step int32, scalars f32");
    hrm::adamw_flat_launch(w.data_ptr<float>(), m_.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr<float>(),
                           w.numel(), (float)lr, (float)wd, (float)b1, (float)b2, (float)eps, step.data_ptr<int>(),
                           scalars.data_ptr<float>(), hrm::gemm_sm_count(), cur_stream());
  });
  m.def("pho_score", [](at::Tensor rec_ids, at::Tensor rec_len, at::Tensor q, at::Tensor scores) {
    c10::cuda::CUDAGuard g(rec_ids.device());
    TORCH_CHECK(rec_ids.is_cuda() && rec_ids.scalar_type() == at::kInt && rec_ids.dim() == 2 && rec_ids.size(1) == 8 &&
                    rec_ids.is_contiguous(), "rec_ids: int32 [n, 8] contiguous on the GPU");
    TORCH_CHECK(rec_len.scalar_type() == at::kInt && rec_len.numel() == rec_ids.size(0), "rec_len: int32 [n]");
    TORCH_CHECK(q.scalar_type() == at::kInt && q.is_cuda() && q.numel() <= 32, "q: int32 [<= 32] on the GPU");
    TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.numel() == rec_ids.size(0), "scores: f32 [n]");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(rec_ids.data_ptr()) & 15) == 0, "rec_ids must be 16-byte aligned");
    hrm::pho_score_launch(reinterpret_cast<const uint32_t*>(rec_ids.data_ptr<int>()),
                          reinterpret_cast<const uint32_t*>(rec_len.data_ptr<int>()),
                          reinterpret_cast<const uint32_t*>(q.data_ptr<int>()), (int)q.numel(),
                          scores.data_ptr<float>(), rec_ids.size(0), hrm::gemm_sm_count(), cur_stream());
  });
  m.def("w8a16_chain", &w8a16_chain, "multi-phase decode GEMM chain in one cooperative launch");
  m.def("chain_phase_plan", &chain_phase_plan_py, "(bn, ws_floats, counters) of one chain phase on all SMs");
  m.def("set_pdl", &hrm::set_pdl_enabled, "programmatic dependent launch of the decode-path kernels on / off");
  m.def("pdl_enabled", &hrm::pdl_enabled);
  m.def("set_gemm_m_fastest", &hrm::set_gemm_m_fastest,
        "m-fastest output-tile numbering for GEMMs with more than one token block on / off");
  m.def("gemm_m_fastest", &hrm::gemm_m_fastest);
  m.def("gemm_tile_walk", &gemm_tile_walk_py, "(n_tile, m_tile, kt) per unit of [u0, u1), flattened",
        py::arg("n_tiles"), py::arg("m_tiles"), py::arg("k_tiles"), py::arg("u0"), py::arg("u1"),
        py::arg("m_fastest"));
  m.def("set_gemm_trace", [](c10::optional<at::Tensor> t) {
    if (t.has_value() && t->defined()) {
      TORCH_CHECK(t->scalar_type() == at::kLong && t->numel() >= 16 * hrm::kGemmTraceLen, "trace: int64[16*1024]");
      hrm::set_gemm_trace(reinterpret_cast<long long*>(t->data_ptr<int64_t>()));
    } else {
      hrm::set_gemm_trace(nullptr);
    }
  });
  m.def("set_status_word", [](at::Tensor t) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt, "status word must be a CUDA int32 tensor");
    hrm::set_status_word(t.device().index(), t.data_ptr<int>());
  });
  hrm::register_comm_bindings(m);
}
