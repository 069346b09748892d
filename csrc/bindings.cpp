// Python bindings of the sm_100a kernels. Every entry point checks device, dtype,
// contiguity and alignment and raises on anything its kernel does not handle, so a
// kernel never receives arguments it was not written for.
#include <torch/extension.h>

#include <map>
#include <utility>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common/tma.h"
#include "gemm/gemm.h"
#include "fused/fused.h"
#include "attn/attn.h"
#include "attn/sla.h"
#include "comm/comm.h"
#include "moe/moe.h"
#include "vae/conv3d.h"
#include "vae/groupnorm.h"

namespace {

void check_cuda_tensor(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16(const torch::Tensor& t, const char* name) {
  check_cuda_tensor(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16");
}
void check_rows(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have unit stride in its last dimension");
  TORCH_CHECK((t.stride(0) * t.element_size()) % 16 == 0, name,
              " row stride must be a multiple of 16 bytes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
}
cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// D = A * B^T with the selected epilogue. `a_t`: A is stored [K, M]; `b_t`: B is [K, N].
void gemm(torch::Tensor A, torch::Tensor B, torch::Tensor D, int64_t epi, bool a_t, bool b_t,
          c10::optional<torch::Tensor> C, c10::optional<torch::Tensor> bias,
          c10::optional<torch::Tensor> D2, c10::optional<torch::Tensor> rope_tab,
          int64_t rope_cols, int64_t rope_rows_per_seq, int64_t rope_pos_offset,
          int64_t rope_head_dim, c10::optional<torch::Tensor> gate,
          int64_t gate_rows_per_group, int64_t splits, int64_t bn,
          c10::optional<torch::Tensor> gb_counters, std::vector<int64_t> gb_peers,
          int64_t gb_rank, int64_t gb_elem0, int64_t gb_shard, int64_t gb_epoch) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_cuda_tensor(D, "D");
  check_rows(A, "A");
  check_rows(B, "B");
  check_rows(D, "D");
  const c10::cuda::CUDAGuard guard(A.device());
  ddb::GemmArgs a;
  a.a_mn_major = a_t;
  a.b_mn_major = b_t;
  a.M = a_t ? A.size(1) : A.size(0);
  a.K = a_t ? A.size(0) : A.size(1);
  a.N = b_t ? B.size(1) : B.size(0);
  const int64_t kb = b_t ? B.size(0) : B.size(1);
  TORCH_CHECK(kb == a.K, "gemm: inner dimensions differ (", a.K, " vs ", kb, ")");
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.D = D.data_ptr();
  a.ldd = D.stride(0);
  TORCH_CHECK(D.size(0) == a.M, "gemm: D has ", D.size(0), " rows, expected ", a.M);
  const bool f32_out = (epi == ddb::kEpiF32 || epi == ddb::kEpiF32Atomic);
  TORCH_CHECK(D.scalar_type() == (f32_out ? torch::kFloat32 : torch::kBFloat16),
              "gemm: D dtype does not match the epilogue");
  int64_t d_cols = a.N;
  if (epi == ddb::kEpiDSwiGLU) d_cols = 2 * a.N;
  TORCH_CHECK(D.size(1) >= d_cols, "gemm: D too narrow");
  if (C) {
    check_bf16(*C, "C");
    check_rows(*C, "C");
    TORCH_CHECK(C->size(0) == a.M, "gemm: C rows");
    a.C = C->data_ptr();
    a.ldc = C->stride(0);
  }
  if (epi == ddb::kEpiDSwiGLU) TORCH_CHECK(C.has_value(), "dswiglu epilogue needs C = gu");
  if (bias) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->is_contiguous() &&
                    bias->numel() >= a.N,
                "gemm: bias must be contiguous fp32 [N]");
    a.bias = bias->data_ptr<float>();
  }
  if (epi == ddb::kEpiSwiGLU) {
    TORCH_CHECK(D2.has_value(), "swiglu epilogue needs D2");
    check_bf16(*D2, "D2");
    check_rows(*D2, "D2");
    TORCH_CHECK(D2->size(0) == a.M && D2->size(1) >= a.N / 2, "gemm: D2 shape");
    a.D2 = D2->data_ptr();
    a.ldd2 = D2->stride(0);
  }
  if (epi == ddb::kEpiRope) {
    TORCH_CHECK(rope_tab.has_value() && rope_tab->scalar_type() == torch::kFloat32 &&
                    rope_tab->is_contiguous(),
                "rope epilogue needs a contiguous fp32 table [P, head_dim/2, 2]");
    TORCH_CHECK(rope_head_dim % 32 == 0, "rope head_dim must be a multiple of 32");
    TORCH_CHECK(rope_cols % rope_head_dim == 0, "rope_cols must be whole heads");
    const int64_t max_pos = rope_tab->numel() / rope_head_dim;
    TORCH_CHECK(rope_pos_offset + std::min<int64_t>(rope_rows_per_seq, a.M) <= max_pos,
                "rope table too short for the requested positions");
    a.rope_tab = reinterpret_cast<const float2*>(rope_tab->data_ptr<float>());
    a.rope_cols = rope_cols;
    a.rope_rows_per_seq = rope_rows_per_seq;
    a.rope_pos_offset = rope_pos_offset;
    a.rope_head_dim = rope_head_dim;
  }
  if (epi == ddb::kEpiGateResidual) {
    TORCH_CHECK(gate.has_value(), "gated residual needs gate");
    check_bf16(*gate, "gate");
    check_rows(*gate, "gate");
    a.gate = gate->data_ptr();
    a.ldg = gate->stride(0);
    a.gate_rows_per_group = gate_rows_per_group;
    TORCH_CHECK((a.M + gate_rows_per_group - 1) / gate_rows_per_group <= gate->size(0),
                "gate has too few rows");
  }
  a.splits = splits;
  a.bn = bn;
  if (gb_counters) {  // FSDP weight all-gather fused into the B loads
    TORCH_CHECK(!b_t, "gemm: the fused weight gather reads a K-major B");
    TORCH_CHECK(gb_counters->is_cuda() && gb_counters->scalar_type() == torch::kInt32 &&
                    gb_counters->is_contiguous() && gb_counters->numel() >= (a.N + 127) / 128,
                "gemm: gather counters must be int32 CUDA [ceil(N / 128)]");
    TORCH_CHECK(!gb_peers.empty() && static_cast<int>(gb_peers.size()) <= ddb::kMaxGemmPeers,
                "gemm: gather peer table");
    a.gb_world = static_cast<int>(gb_peers.size());
    a.gb_rank = static_cast<int>(gb_rank);
    a.gb_elem0 = gb_elem0;
    a.gb_shard = gb_shard;
    a.gb_epoch = static_cast<unsigned>(gb_epoch);
    a.gb_counters = reinterpret_cast<unsigned*>(gb_counters->data_ptr<int>());
    for (size_t r = 0; r < gb_peers.size(); ++r)
      a.gb_peers[r] = reinterpret_cast<const void*>(gb_peers[r]);
  }
  ddb::gemm(a, static_cast<int>(epi), stream());
}

int64_t read_status() {
  int dev = 0;
  ddb::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  int v = 0;
  ddb::check_cuda(cudaMemcpy(&v, ddb::device_status(dev), sizeof(int), cudaMemcpyDeviceToHost),
                  "read status");
  return v;
}
int64_t read_status_index() {
  int dev = 0;
  ddb::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  int v[2] = {0, 0};
  ddb::check_cuda(cudaMemcpy(v, ddb::device_status(dev), sizeof(v), cudaMemcpyDeviceToHost),
                  "read status");
  return v[1];
}
void reset_status() {
  int dev = 0;
  ddb::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  ddb::check_cuda(cudaMemset(ddb::device_status(dev), 0, 2 * sizeof(int)), "reset status");
}

// ------------------------------------------------------------------ fused norm
std::vector<torch::Tensor> adaln_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor mod,
                                     int64_t scale_off, int64_t shift_off,
                                     int64_t rows_per_group, double eps) {
  check_bf16(x, "x");
  check_rows(x, "x");
  TORCH_CHECK(x.is_contiguous(), "x must be contiguous");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.numel() == x.size(1),
              "w must be fp32 [D]");
  TORCH_CHECK(mod.scalar_type() == torch::kFloat32 && mod.dim() == 2 && mod.stride(1) == 1,
              "mod must be fp32 [groups, cols]");
  TORCH_CHECK(mod.stride(0) % 4 == 0 && scale_off % 4 == 0 && shift_off % 4 == 0,
              "mod columns must be 16-byte aligned");
  const int64_t M = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 256 == 0 && D <= 2048 && D != 1280 && D != 1792,
              "adaln: D must be 256, 512, 768, 1024, 1536 or 2048");
  TORCH_CHECK((M + rows_per_group - 1) / rows_per_group <= mod.size(0), "mod has too few rows");
  TORCH_CHECK(std::max(scale_off, shift_off) + D <= mod.size(1), "mod too narrow");
  const c10::cuda::CUDAGuard guard(x.device());
  auto h = torch::empty_like(x);
  auto rstd = torch::empty({M}, x.options().dtype(torch::kFloat32));
  ddb::AdaLNArgs a;
  a.M = M; a.D = D; a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.w = w.data_ptr<float>(); a.mod = mod.data_ptr<float>(); a.ld_mod = mod.stride(0);
  a.scale_off = scale_off; a.shift_off = shift_off; a.rows_per_group = rows_per_group;
  a.eps = static_cast<float>(eps);
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr()); a.rstd = rstd.data_ptr<float>();
  ddb::adaln_rmsnorm_fwd(a, stream());
  return {h, rstd};
}

torch::Tensor adaln_bwd(torch::Tensor dh, torch::Tensor x, torch::Tensor rstd, torch::Tensor w,
                        torch::Tensor mod, int64_t scale_off, int64_t shift_off,
                        int64_t rows_per_group, c10::optional<torch::Tensor> dres,
                        c10::optional<torch::Tensor> dw, torch::Tensor dmod) {
  check_bf16(dh, "dh");
  check_bf16(x, "x");
  TORCH_CHECK(dh.is_contiguous() && x.is_contiguous() && dh.sizes() == x.sizes(), "dh/x shape");
  const int64_t M = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 256 == 0 && D <= 2048 && D != 1280 && D != 1792,
              "adaln bwd: D must be 256, 512, 768, 1024, 1536 or 2048");
  TORCH_CHECK(rstd.scalar_type() == torch::kFloat32 && rstd.numel() == M, "rstd");
  TORCH_CHECK(dmod.scalar_type() == torch::kFloat32 && dmod.dim() == 2 && dmod.stride(1) == 1 &&
                  dmod.size(0) >= (M + rows_per_group - 1) / rows_per_group,
              "dmod must be fp32 [groups, cols]");
  TORCH_CHECK(mod.stride(0) % 4 == 0 && mod.scalar_type() == torch::kFloat32, "mod");
  const c10::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  ddb::AdaLNArgs a;
  a.M = M; a.D = D; a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.w = w.data_ptr<float>(); a.mod = mod.data_ptr<float>(); a.ld_mod = mod.stride(0);
  a.scale_off = scale_off; a.shift_off = shift_off; a.rows_per_group = rows_per_group;
  a.rstd = rstd.data_ptr<float>();
  a.dh = reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr());
  if (dres) {
    check_bf16(*dres, "dres");
    TORCH_CHECK(dres->is_contiguous() && dres->sizes() == x.sizes(), "dres shape");
    a.dres = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
  }
  a.dx = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  if (dw) {
    TORCH_CHECK(dw->scalar_type() == torch::kFloat32 && dw->is_contiguous() && dw->numel() == D, "dw");
    a.dw = dw->data_ptr<float>();
  }
  a.dmod = dmod.data_ptr<float>(); a.ld_dmod = dmod.stride(0);
  ddb::adaln_rmsnorm_bwd(a, stream());
  return dx;
}

// ------------------------------------------------------------------ optimizer / casts
void adamw_flat(torch::Tensor master, torch::Tensor grad, torch::Tensor m, torch::Tensor v,
                c10::optional<torch::Tensor> compute, torch::Tensor clip, double lr, double b1,
                double b2, double eps, double wd, double bc1, double bc2, double grad_scale,
                int64_t decay_end) {
  for (auto* t : {&master, &grad, &m, &v}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous(),
                "adamw buffers must be contiguous fp32 CUDA tensors");
    TORCH_CHECK(t->numel() == master.numel(), "adamw buffers differ in length");
  }
  TORCH_CHECK(clip.scalar_type() == torch::kFloat32 && clip.numel() == 1 && clip.is_cuda(), "clip");
  const c10::cuda::CUDAGuard guard(master.device());
  ddb::AdamWArgs a;
  a.master = master.data_ptr<float>(); a.grad = grad.data_ptr<float>();
  a.m = m.data_ptr<float>(); a.v = v.data_ptr<float>();
  if (compute) {
    check_bf16(*compute, "compute");
    TORCH_CHECK(compute->numel() == master.numel() && compute->is_contiguous(), "compute");
    a.compute = reinterpret_cast<__nv_bfloat16*>(compute->data_ptr());
  }
  a.clip = clip.data_ptr<float>();
  a.n = master.numel(); a.decay_end = decay_end;
  a.lr = lr; a.b1 = b1; a.b2 = b2; a.eps = eps; a.wd = wd; a.bc1 = bc1; a.bc2 = bc2;
  a.grad_scale = grad_scale;
  ddb::adamw_flat(a, stream());
}

void cast_bf16(torch::Tensor src, torch::Tensor dst) {
  TORCH_CHECK(src.scalar_type() == torch::kFloat32 && src.is_contiguous() && src.is_cuda(), "src");
  check_bf16(dst, "dst");
  TORCH_CHECK(dst.numel() == src.numel() && dst.is_contiguous(), "dst");
  const c10::cuda::CUDAGuard guard(src.device());
  ddb::cast_f32_bf16(src.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()),
                     src.numel(), stream());
}

torch::Tensor sq_norm(torch::Tensor x) {
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.is_cuda(), "x");
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::zeros({}, x.options());
  ddb::sq_norm_f32(x.data_ptr<float>(), x.numel(), out.data_ptr<float>(), stream());
  return out;
}

void rope_rotate(torch::Tensor x, int64_t rot_cols, torch::Tensor tab, int64_t head_dim,
                 int64_t rows_per_seq, int64_t pos_offset, bool inverse) {
  check_bf16(x, "x");
  check_rows(x, "x");
  TORCH_CHECK(rot_cols % head_dim == 0 && head_dim % 8 == 0, "rope_rotate: columns");
  TORCH_CHECK(tab.scalar_type() == torch::kFloat32 && tab.is_contiguous(), "tab");
  TORCH_CHECK(pos_offset + std::min<int64_t>(rows_per_seq, x.size(0)) <= tab.numel() / head_dim,
              "rope table too short");
  const c10::cuda::CUDAGuard guard(x.device());
  ddb::rope_rotate_bf16(reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), x.size(0),
                        rot_cols, reinterpret_cast<const float2*>(tab.data_ptr<float>()), head_dim,
                        rows_per_seq, pos_offset, inverse, stream());
}

// ------------------------------------------------------------------ attention
ddb::AttnArgs make_attn_args(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                             int64_t q_col, int64_t k_col, int64_t v_col, int64_t B, int64_t H,
                             int64_t Tq, int64_t S, int64_t q_rows_per_b, int64_t kv_rows_per_b,
                             int64_t causal, int64_t tpf, int64_t q_pos_offset,
                             int64_t kv_pos_offset, double scale) {
  for (auto* t : {&q, &k, &v}) {
    check_bf16(*t, "q/k/v");
    check_rows(*t, "q/k/v");
  }
  TORCH_CHECK(q.size(0) >= (B - 1) * q_rows_per_b + Tq &&
                  k.size(0) >= (B - 1) * kv_rows_per_b + S &&
                  v.size(0) >= (B - 1) * kv_rows_per_b + S,
              "attention: tensors have fewer rows than the samples need");
  TORCH_CHECK(k.size(0) == v.size(0), "attention: k and v differ in rows");
  TORCH_CHECK(q_col + H * 64 <= q.size(1) && k_col + H * 64 <= k.size(1) &&
                  v_col + H * 64 <= v.size(1),
              "attention: head columns out of range");
  TORCH_CHECK(q_col % 8 == 0 && k_col % 8 == 0 && v_col % 8 == 0, "attention: column offsets");
  TORCH_CHECK(tpf >= 1, "tokens per frame");
  ddb::AttnArgs a;
  a.B = B; a.H = H; a.Tq = Tq; a.S = S; a.q_rows_per_b = q_rows_per_b;
  a.kv_rows_per_b = kv_rows_per_b;
  a.q = q.data_ptr(); a.ldq = q.stride(0); a.q_col = q_col;
  a.k = k.data_ptr(); a.ldk = k.stride(0); a.k_col = k_col;
  a.v = v.data_ptr(); a.ldv = v.stride(0); a.v_col = v_col;
  a.causal = causal; a.tpf = tpf; a.q_pos_offset = q_pos_offset;
  a.kv_pos_offset = kv_pos_offset; a.scale = static_cast<float>(scale);
  a.q_rows_total = q.size(0);
  a.kv_rows_total = k.size(0);
  return a;
}

// split-KV override for tests: 0 = chosen per launch, n >= 1 = always n splits
int64_t g_attn_kv_splits = 0;

void attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
              c10::optional<torch::Tensor> lse, int64_t q_col, int64_t k_col, int64_t v_col,
              int64_t o_col, int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t q_rows_per_b,
              int64_t kv_rows_per_b, int64_t causal, int64_t tpf, int64_t q_pos_offset,
              int64_t kv_pos_offset, double scale, c10::optional<torch::Tensor> pair_blocks,
              c10::optional<torch::Tensor> pair_mask, c10::optional<torch::Tensor> pair_count) {
  const c10::cuda::CUDAGuard guard(q.device());
  auto a = make_attn_args(q, k, v, q_col, k_col, v_col, B, H, Tq, S, q_rows_per_b, kv_rows_per_b,
                          causal, tpf, q_pos_offset, kv_pos_offset, scale);
  check_bf16(o, "o");
  check_rows(o, "o");
  TORCH_CHECK(o.size(0) >= (B - 1) * q_rows_per_b + Tq && o_col + H * 64 <= o.size(1), "o shape");
  a.o = o.data_ptr(); a.ldo = o.stride(0); a.o_col = o_col;
  if (lse) {
    TORCH_CHECK(lse->scalar_type() == torch::kFloat32 && lse->is_contiguous() &&
                    lse->numel() >= B * H * Tq, "lse must be fp32 [B, H, Tq]");
    a.lse = lse->data_ptr<float>();
  }
  if (pair_count) {
    TORCH_CHECK(pair_blocks && pair_mask, "sparse attention needs blocks, mask and count");
    const int64_t nqt = (Tq + 127) / 128;
    TORCH_CHECK(pair_count->scalar_type() == torch::kInt32 && pair_count->numel() == B * H * nqt,
                "pair_count must be int32 [B*H*n_qtiles]");
    TORCH_CHECK(pair_blocks->scalar_type() == torch::kInt32 && pair_blocks->dim() == 2 &&
                    pair_blocks->size(0) == B * H * nqt && pair_blocks->is_contiguous(),
                "pair_blocks must be int32 [B*H*n_qtiles, max_pairs]");
    TORCH_CHECK(pair_mask->scalar_type() == torch::kUInt8 && pair_mask->sizes() == pair_blocks->sizes() &&
                    pair_mask->is_contiguous(), "pair_mask must be uint8 like pair_blocks");
    a.pair_blocks = pair_blocks->data_ptr<int>();
    a.pair_mask = pair_mask->data_ptr<uint8_t>();
    a.pair_count = pair_count->data_ptr<int>();
    a.max_pairs = pair_blocks->size(1);
  }
  // split-KV when the grid would leave SMs idle (scratch from the caching allocator)
  const int splits = g_attn_kv_splits > 0 ? (a.pair_count ? 1 : static_cast<int>(g_attn_kv_splits))
                                          : ddb::attn_fwd_kv_splits(a);
  if (splits > 1) {
    long oe = 0, le = 0;
    ddb::attn_fwd_split_scratch(a, splits, &oe, &le);
    // one persistent scratch per (device, stream), grown on demand: launches on one
    // stream run in order, so reusing it needs no allocation per call
    // (never destroyed: tensors released after the CUDA context at exit would fault)
    static auto* scratch = new std::map<std::pair<int, cudaStream_t>, torch::Tensor>();
    const auto key = std::make_pair(static_cast<int>(q.get_device()), stream());
    torch::Tensor& buf = (*scratch)[key];
    const long need = (oe + 63) / 64 * 64 + le;
    if (!buf.defined() || buf.numel() < need)
      buf = torch::empty({need}, q.options().dtype(torch::kFloat32));
    a.kv_splits = splits;
    a.o_part = buf.data_ptr<float>();
    a.lse_part = a.o_part + (oe + 63) / 64 * 64;
  }
  ddb::attn_fwd(a, stream());
}

void attn_fwd_set_trace(c10::optional<torch::Tensor> trace, int64_t cta) {
  if (trace) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == torch::kInt64 && trace->numel() >= 3 * 8 * 64,
                "trace must be int64 CUDA [3 * 8 * 64]");
    ddb::attn_fwd_set_trace(reinterpret_cast<long long*>(trace->data_ptr<int64_t>()), cta);
  } else {
    ddb::attn_fwd_set_trace(nullptr, 0);
  }
}

void attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
              torch::Tensor dout, torch::Tensor lse, torch::Tensor delta, torch::Tensor dq_acc,
              torch::Tensor dk, torch::Tensor dv, int64_t q_col, int64_t k_col, int64_t v_col,
              int64_t o_col, int64_t do_col, int64_t dk_col, int64_t dv_col, int64_t B, int64_t H,
              int64_t Tq, int64_t S, int64_t q_rows_per_b, int64_t kv_rows_per_b, int64_t causal,
              int64_t tpf, int64_t q_pos_offset, int64_t kv_pos_offset, double scale,
              c10::optional<torch::Tensor> kv_qtiles, c10::optional<torch::Tensor> kv_qmask,
              c10::optional<torch::Tensor> kv_count, int64_t debug_flags,
              c10::optional<torch::Tensor> trace, int64_t trace_cta) {
  const c10::cuda::CUDAGuard guard(q.device());
  ddb::AttnBwdArgs g;
  g.debug_flags = debug_flags;
  if (trace) {
    TORCH_CHECK(trace->scalar_type() == torch::kInt64 && trace->numel() >= 4 * 8 * 64, "trace");
    g.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
    g.trace_cta = trace_cta;
  }
  g.f = make_attn_args(q, k, v, q_col, k_col, v_col, B, H, Tq, S, q_rows_per_b, kv_rows_per_b,
                       causal, tpf, q_pos_offset, kv_pos_offset, scale);
  check_bf16(dout, "dout");
  check_rows(dout, "dout");
  TORCH_CHECK(dout.size(0) >= B * q_rows_per_b && do_col + H * 64 <= dout.size(1), "dout shape");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.numel() >= B * H * Tq, "lse");
  TORCH_CHECK(delta.scalar_type() == torch::kFloat32 && delta.numel() >= B * H * Tq, "delta");
  TORCH_CHECK(dq_acc.scalar_type() == torch::kFloat32 && dq_acc.dim() == 2 &&
                  dq_acc.stride(1) == 1 && dq_acc.stride(0) % 4 == 0 &&
                  dq_acc.size(0) >= B * q_rows_per_b && dq_acc.size(1) >= H * 64,
              "dq_acc must be fp32 [rows, >= H*64]");
  for (auto* t : {&dk, &dv}) {
    check_bf16(*t, "dk/dv");
    check_rows(*t, "dk/dv");
    TORCH_CHECK(t->size(0) >= B * kv_rows_per_b, "dk/dv rows");
  }
  TORCH_CHECK(dk_col + H * 64 <= dk.size(1) && dv_col + H * 64 <= dv.size(1), "dk/dv columns");
  g.f.lse = lse.data_ptr<float>();
  g.f.o = o.data_ptr(); g.f.ldo = o.stride(0); g.f.o_col = o_col;
  g.dout = dout.data_ptr(); g.lddo = dout.stride(0); g.do_col = do_col;
  g.delta = delta.data_ptr<float>();
  g.dq_acc = dq_acc.data_ptr<float>(); g.ld_dqacc = dq_acc.stride(0);
  g.dk = dk.data_ptr(); g.lddk = dk.stride(0); g.dk_col = dk_col;
  g.dv = dv.data_ptr(); g.lddv = dv.stride(0); g.dv_col = dv_col;
  if (kv_count) {
    TORCH_CHECK(kv_qtiles && kv_qmask, "sparse backward needs q-tile lists, masks and counts");
    const int64_t nkt = (S + 127) / 128;
    TORCH_CHECK(kv_count->scalar_type() == torch::kInt32 && kv_count->numel() == B * H * nkt,
                "kv_count must be int32 [B*H*n_kvtiles]");
    TORCH_CHECK(kv_qtiles->scalar_type() == torch::kInt32 && kv_qtiles->dim() == 2 &&
                    kv_qtiles->size(0) == B * H * nkt && kv_qtiles->is_contiguous(), "kv_qtiles");
    TORCH_CHECK(kv_qmask->scalar_type() == torch::kUInt8 && kv_qmask->sizes() == kv_qtiles->sizes() &&
                    kv_qmask->is_contiguous(), "kv_qmask");
    g.kv_qtiles = kv_qtiles->data_ptr<int>();
    g.kv_qmask = kv_qmask->data_ptr<uint8_t>();
    g.kv_count = kv_count->data_ptr<int>();
    g.max_q = kv_qtiles->size(1);
  }
  ddb::attn_bwd(g, stream());
}

void attn_delta(torch::Tensor o, torch::Tensor dout, torch::Tensor delta, int64_t o_col,
                int64_t do_col, int64_t B, int64_t H, int64_t Tq, int64_t rows_per_b) {
  check_bf16(o, "o");
  check_bf16(dout, "dout");
  check_rows(o, "o");
  check_rows(dout, "dout");
  TORCH_CHECK(delta.scalar_type() == torch::kFloat32 && delta.numel() >= B * H * Tq, "delta");
  const c10::cuda::CUDAGuard guard(o.device());
  ddb::attn_bwd_delta(o.data_ptr(), o.stride(0), o_col, dout.data_ptr(), dout.stride(0), do_col,
                      delta.data_ptr<float>(), B, H, Tq, rows_per_b, stream());
}

void attn_dq_finalize(torch::Tensor dq_acc, torch::Tensor dq, int64_t dq_col, int64_t H,
                      c10::optional<torch::Tensor> rope_tab, int64_t rows_per_seq,
                      int64_t pos_offset) {
  TORCH_CHECK(dq_acc.scalar_type() == torch::kFloat32 && dq_acc.stride(1) == 1 &&
                  dq_acc.stride(0) % 4 == 0, "dq_acc");
  check_bf16(dq, "dq");
  check_rows(dq, "dq");
  TORCH_CHECK(dq.size(0) == dq_acc.size(0) && dq_col + H * 64 <= dq.size(1), "dq shape");
  const float2* tab = nullptr;
  if (rope_tab) {
    TORCH_CHECK(rope_tab->scalar_type() == torch::kFloat32 && rope_tab->is_contiguous() &&
                    rope_tab->numel() >= (pos_offset + std::min<int64_t>(rows_per_seq, dq.size(0))) * 64,
                "rope table");
    tab = reinterpret_cast<const float2*>(rope_tab->data_ptr<float>());
  }
  const c10::cuda::CUDAGuard guard(dq.device());
  ddb::attn_dq_finalize(dq_acc.data_ptr<float>(), dq_acc.stride(0), dq.data_ptr(), dq.stride(0),
                        dq_col, dq.size(0), H, tab, rows_per_seq, pos_offset, stream());
}

// ------------------------------------------------------------------ batched GEMM
// D[b] = A[b] B[b]^T for 3-D bf16 A, B (row-major per batch); D is [batch * M, N].
// Tensor-parallel forms of the GEMM: the all-gather of A fused into its TMA loads (rows of
// peer p read from a_peers[p]) and/or the reduce-scatter fused into the bf16 store (row r
// stored into rank r / d_rows_per_peer's buffer through the device pointer table d_peers).
void gemm_tp(torch::Tensor A, torch::Tensor B, c10::optional<torch::Tensor> D, int64_t epi, int64_t M,
             std::vector<int64_t> a_peers, int64_t a_rows_per_peer, c10::optional<torch::Tensor> d_peers,
             int64_t d_rows_per_peer, int64_t d_slot, int64_t ldd, c10::optional<torch::Tensor> D2,
             c10::optional<torch::Tensor> rope_tab, int64_t rope_cols, int64_t rope_rows_per_seq,
             int64_t rope_pos_offset, int64_t rope_head_dim) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_rows(A, "A");
  check_rows(B, "B");
  const c10::cuda::CUDAGuard guard(A.device());
  ddb::GemmArgs a;
  a.M = M;
  a.K = A.size(1);
  a.N = B.size(0);
  TORCH_CHECK(B.size(1) == a.K, "gemm_tp: inner dimensions differ");
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  if (!a_peers.empty()) {
    TORCH_CHECK(static_cast<int>(a_peers.size()) <= ddb::kMaxGemmPeers, "gemm_tp: too many peers");
    a.a_npeers = static_cast<int>(a_peers.size());
    a.a_rows_per_peer = a_rows_per_peer;
    for (size_t p = 0; p < a_peers.size(); ++p) a.a_peer_ptrs[p] = reinterpret_cast<const void*>(a_peers[p]);
  } else {
    TORCH_CHECK(A.size(0) == M, "gemm_tp: A rows");
  }
  if (d_peers) {
    TORCH_CHECK(d_peers->is_cuda() && d_peers->scalar_type() == torch::kInt64, "gemm_tp: d_peers table");
    TORCH_CHECK(epi == ddb::kEpiBf16, "gemm_tp: the reduce-scatter store is bf16 only");
    a.d_peers = reinterpret_cast<void* const*>(d_peers->data_ptr<int64_t>());
    a.d_rows_per_peer = d_rows_per_peer;
    a.d_slot = d_slot;
    a.ldd = ldd;
    a.D = reinterpret_cast<void*>(1);  // never written through: rows go to the peers
  } else {
    TORCH_CHECK(D.has_value(), "gemm_tp: D or d_peers");
    check_bf16(*D, "D");
    check_rows(*D, "D");
    TORCH_CHECK(D->size(0) == M, "gemm_tp: D rows");
    a.D = D->data_ptr();
    a.ldd = D->stride(0);
  }
  if (epi == ddb::kEpiSwiGLU) {
    TORCH_CHECK(D2.has_value(), "swiglu epilogue needs D2");
    check_bf16(*D2, "D2");
    a.D2 = D2->data_ptr();
    a.ldd2 = D2->stride(0);
  }
  if (epi == ddb::kEpiRope) {
    TORCH_CHECK(rope_tab.has_value() && rope_tab->scalar_type() == torch::kFloat32, "rope table");
    a.rope_tab = reinterpret_cast<const float2*>(rope_tab->data_ptr<float>());
    a.rope_cols = rope_cols;
    a.rope_rows_per_seq = rope_rows_per_seq;
    a.rope_pos_offset = rope_pos_offset;
    a.rope_head_dim = rope_head_dim;
  }
  ddb::gemm(a, static_cast<int>(epi), stream());
}

// out[r] = residual[r] + sum_s recv[s * rows + r] (bf16, fp32 accumulation)
// out [n] = residual + sum over ranks of their bf16 partial buffers (peer pointer table)
torch::Tensor tp_allreduce_sum(torch::Tensor peer_table, int64_t world, int64_t n, torch::Tensor like,
                               c10::optional<torch::Tensor> residual) {
  TORCH_CHECK(peer_table.is_cuda() && peer_table.scalar_type() == torch::kInt64 && peer_table.numel() >= world,
              "tp_allreduce_sum: peer table must be int64 CUDA [world]");
  check_bf16(like, "like");
  TORCH_CHECK(like.numel() == n && like.is_contiguous(), "tp_allreduce_sum: like must be contiguous with n elements");
  auto out = torch::empty_like(like);
  const __nv_bfloat16* res = nullptr;
  if (residual) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->numel() == n && residual->is_contiguous(), "tp_allreduce_sum: residual shape");
    res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  ddb::tp_allreduce_sum(reinterpret_cast<const __nv_bfloat16* const*>(peer_table.data_ptr<int64_t>()), world, n,
                        res, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), stream());
  return out;
}

torch::Tensor tp_sum_rows(torch::Tensor recv, int64_t world, int64_t rows, c10::optional<torch::Tensor> residual) {
  check_bf16(recv, "recv");
  TORCH_CHECK(recv.is_contiguous() && recv.size(0) >= world * rows, "recv [world * rows, d]");
  const c10::cuda::CUDAGuard guard(recv.device());
  const int64_t d = recv.size(1);
  auto out = torch::empty({rows, d}, recv.options());
  const __nv_bfloat16* res = nullptr;
  if (residual) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->is_contiguous() && residual->size(0) == rows && residual->size(1) == d, "residual");
    res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  ddb::tp_sum_rows(reinterpret_cast<const __nv_bfloat16*>(recv.data_ptr()), world, rows, d, res,
                   reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), stream());
  return out;
}

void gemm_batched(torch::Tensor A, torch::Tensor B, torch::Tensor D, int64_t epi, bool a_t,
                  bool b_t) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3 && A.size(0) == B.size(0), "gemm_batched: 3-D A, B");
  TORCH_CHECK(A.stride(2) == 1 && B.stride(2) == 1, "gemm_batched: unit inner stride");
  TORCH_CHECK((A.stride(1) * 2) % 16 == 0 && (B.stride(1) * 2) % 16 == 0, "gemm_batched: row strides");
  check_rows(D, "D");
  const c10::cuda::CUDAGuard guard(A.device());
  ddb::GemmArgs a;
  a.batch = A.size(0);
  a.a_mn_major = a_t;
  a.b_mn_major = b_t;
  a.M = a_t ? A.size(2) : A.size(1);
  a.K = a_t ? A.size(1) : A.size(2);
  a.N = b_t ? B.size(2) : B.size(1);
  TORCH_CHECK((b_t ? B.size(1) : B.size(2)) == a.K, "gemm_batched: inner dimensions differ");
  a.A = A.data_ptr(); a.lda = A.stride(1); a.stride_a = A.stride(0);
  a.B = B.data_ptr(); a.ldb = B.stride(1); a.stride_b = B.stride(0);
  a.D = D.data_ptr(); a.ldd = D.stride(0);
  TORCH_CHECK(D.size(0) == static_cast<int64_t>(a.batch) * a.M && D.size(1) >= a.N, "gemm_batched: D shape");
  const bool f32_out = (epi == ddb::kEpiF32 || epi == ddb::kEpiF32Atomic);
  TORCH_CHECK(D.scalar_type() == (f32_out ? torch::kFloat32 : torch::kBFloat16), "gemm_batched: D dtype");
  TORCH_CHECK(epi == ddb::kEpiF32 || epi == ddb::kEpiBf16, "gemm_batched: plain epilogues only");
  ddb::gemm(a, static_cast<int>(epi), stream());
}

// ------------------------------------------------------------------ SLA
void sla_pool(torch::Tensor qkv, torch::Tensor qm, torch::Tensor km, int64_t B, int64_t T, int64_t H) {
  check_bf16(qkv, "qkv");
  check_rows(qkv, "qkv");
  TORCH_CHECK(T % 64 == 0 && qkv.size(0) == B * T && qkv.size(1) >= 3 * H * 64, "sla_pool: qkv shape");
  TORCH_CHECK(qm.scalar_type() == torch::kFloat32 && qm.is_contiguous() && qm.numel() == B * H * T, "qm");
  TORCH_CHECK(km.scalar_type() == torch::kFloat32 && km.is_contiguous() && km.numel() == B * H * T, "km");
  const c10::cuda::CUDAGuard guard(qkv.device());
  ddb::sla_pool(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), B, T, H,
                qm.data_ptr<float>(), km.data_ptr<float>(), stream());
}

void sla_route(torch::Tensor qm, torch::Tensor km, int64_t BH, int64_t nb, int64_t topk,
               int64_t causal, int64_t bpf, bool always_diag, torch::Tensor wlin,
               torch::Tensor pair_blocks, torch::Tensor pair_mask, torch::Tensor pair_count,
               torch::Tensor kv_qtiles, torch::Tensor kv_qmask, torch::Tensor kv_count,
               c10::optional<torch::Tensor> sel_bits) {
  TORCH_CHECK(nb % 2 == 0 && nb <= 256 && nb >= 2, "sla_route: even number of blocks <= 256");
  TORCH_CHECK(qm.numel() == BH * nb * 64 && km.numel() == BH * nb * 64, "sla_route: qm/km");
  check_bf16(wlin, "wlin");
  TORCH_CHECK(wlin.numel() == BH * nb * nb && wlin.is_contiguous(), "wlin");
  const int64_t nt = nb / 2;
  TORCH_CHECK(pair_blocks.scalar_type() == torch::kInt32 && pair_blocks.size(0) == BH * nt &&
                  pair_blocks.is_contiguous(), "pair_blocks");
  TORCH_CHECK(pair_mask.scalar_type() == torch::kUInt8 && pair_mask.sizes() == pair_blocks.sizes(), "pair_mask");
  TORCH_CHECK(pair_count.scalar_type() == torch::kInt32 && pair_count.numel() == BH * nt, "pair_count");
  TORCH_CHECK(kv_qtiles.scalar_type() == torch::kInt32 && kv_qtiles.numel() == BH * nt * nt, "kv_qtiles");
  TORCH_CHECK(kv_qmask.scalar_type() == torch::kUInt8 && kv_qmask.numel() == BH * nt * nt, "kv_qmask");
  TORCH_CHECK(kv_count.scalar_type() == torch::kInt32 && kv_count.numel() == BH * nt, "kv_count");
  const c10::cuda::CUDAGuard guard(qm.device());
  ddb::SlaRouteArgs a;
  a.qm = qm.data_ptr<float>(); a.km = km.data_ptr<float>();
  a.nb = nb; a.topk = topk; a.causal = causal; a.bpf = bpf; a.always_diag = always_diag;
  a.wlin = reinterpret_cast<__nv_bfloat16*>(wlin.data_ptr());
  a.pair_blocks = pair_blocks.data_ptr<int>(); a.pair_mask = pair_mask.data_ptr<uint8_t>();
  a.pair_count = pair_count.data_ptr<int>(); a.max_pairs = pair_blocks.size(1);
  a.kv_qtiles = kv_qtiles.data_ptr<int>(); a.kv_qmask = kv_qmask.data_ptr<uint8_t>();
  a.kv_count = kv_count.data_ptr<int>();
  if (sel_bits) {
    TORCH_CHECK(sel_bits->numel() == BH * nb * ((nb + 31) / 32), "sel_bits");
    a.sel_bits = reinterpret_cast<uint32_t*>(sel_bits->data_ptr<int>());
  }
  ddb::sla_route(a, BH, stream());
}

void sla_kv_state(torch::Tensor qkv, torch::Tensor kvz, int64_t B, int64_t T, int64_t H) {
  check_bf16(qkv, "qkv");
  check_rows(qkv, "qkv");
  check_bf16(kvz, "kvz");
  TORCH_CHECK(kvz.is_contiguous() && kvz.numel() == B * H * (T / 64) * 4160, "kvz");
  const c10::cuda::CUDAGuard guard(qkv.device());
  ddb::sla_kv_state(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), B, T, H,
                    reinterpret_cast<__nv_bfloat16*>(kvz.data_ptr()), stream());
}

void sla_lin_out(torch::Tensor qkv, torch::Tensor state, torch::Tensor o, torch::Tensor den,
                 int64_t B, int64_t T, int64_t H, double eps) {
  check_bf16(qkv, "qkv");
  check_bf16(o, "o");
  check_rows(o, "o");
  TORCH_CHECK(state.scalar_type() == torch::kFloat32 && state.is_contiguous() &&
                  state.numel() == B * H * (T / 64) * 4160, "state");
  TORCH_CHECK(den.scalar_type() == torch::kFloat32 && den.numel() == B * H * T, "den");
  const c10::cuda::CUDAGuard guard(qkv.device());
  ddb::sla_lin_out(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), B, T, H,
                   state.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), o.stride(0),
                   den.data_ptr<float>(), static_cast<float>(eps), stream());
}

void sla_lin_bwd_q(torch::Tensor qkv, torch::Tensor state, torch::Tensor o, torch::Tensor dout,
                   torch::Tensor den, torch::Tensor dsz, torch::Tensor dqkv, int64_t B, int64_t T,
                   int64_t H) {
  for (auto* t : {&qkv, &o, &dout, &dqkv}) check_bf16(*t, "bf16 operand");
  check_bf16(dsz, "dsz");
  TORCH_CHECK(dsz.is_contiguous() && dsz.numel() == B * H * (T / 64) * 4160, "dsz");
  TORCH_CHECK(state.scalar_type() == torch::kFloat32 && state.numel() == B * H * (T / 64) * 4160, "state");
  const c10::cuda::CUDAGuard guard(qkv.device());
  ddb::sla_lin_bwd_q(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), B, T, H,
                     state.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
                     o.stride(0), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                     dout.stride(0), den.data_ptr<float>(),
                     reinterpret_cast<__nv_bfloat16*>(dsz.data_ptr()),
                     reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dqkv.stride(0), stream());
}

void sla_lin_bwd_kv(torch::Tensor qkv, torch::Tensor dkvz, torch::Tensor dqkv, int64_t B, int64_t T,
                    int64_t H) {
  check_bf16(qkv, "qkv");
  check_bf16(dqkv, "dqkv");
  TORCH_CHECK(dkvz.scalar_type() == torch::kFloat32 && dkvz.numel() == B * H * (T / 64) * 4160, "dkvz");
  const c10::cuda::CUDAGuard guard(qkv.device());
  ddb::sla_lin_bwd_kv(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), B, T, H,
                      dkvz.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
                      dqkv.stride(0), stream());
}

// ------------------------------------------------------------------ peer memory
py::tuple ipc_alloc(int64_t bytes) {
  auto a = ddb::ipc_alloc(static_cast<size_t>(bytes));
  return py::make_tuple(reinterpret_cast<int64_t>(a.ptr), py::bytes(a.handle));
}
int64_t ipc_open(py::bytes handle) {
  return reinterpret_cast<int64_t>(ddb::ipc_open(std::string(handle)));
}
void ipc_close(int64_t p) { ddb::ipc_close(reinterpret_cast<void*>(p)); }
void ipc_free(int64_t p) { ddb::ipc_free(reinterpret_cast<void*>(p)); }

// A tensor viewing `numel` elements at a device pointer this extension owns (no copy).
torch::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, torch::Dtype dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {}, opts);
}

void xrank_barrier(torch::Tensor peer_table, int64_t local_ptr, int64_t rank, int64_t world,
                   int64_t epoch, c10::optional<torch::Tensor> payload) {
  TORCH_CHECK(peer_table.is_cuda() && peer_table.scalar_type() == torch::kInt64 &&
                  peer_table.numel() == world, "peer table must be int64 [world] on the device");
  const float* pay = nullptr;
  if (payload) {
    TORCH_CHECK(payload->scalar_type() == torch::kFloat32 && payload->is_cuda(), "payload");
    pay = payload->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(peer_table.device());
  int dev = peer_table.device().index();
  ddb::xrank_barrier(reinterpret_cast<void* const*>(peer_table.data_ptr<int64_t>()),
                     reinterpret_cast<void*>(local_ptr), rank, world, static_cast<uint32_t>(epoch),
                     pay, ddb::device_status(dev), stream());
}

void rs_sum_sqnorm(torch::Tensor grad_table, int64_t world, int64_t off, int64_t len,
                   torch::Tensor red, torch::Tensor sumsq) {
  TORCH_CHECK(grad_table.scalar_type() == torch::kInt64 && grad_table.numel() == world, "grad table");
  TORCH_CHECK(red.scalar_type() == torch::kFloat32 && red.numel() >= len && red.is_contiguous(), "red");
  TORCH_CHECK(sumsq.scalar_type() == torch::kFloat32 && sumsq.numel() >= 1, "sumsq");
  const c10::cuda::CUDAGuard guard(red.device());
  ddb::rs_sum_sqnorm(reinterpret_cast<const float* const*>(grad_table.data_ptr<int64_t>()), world, off,
                     len, red.data_ptr<float>(), sumsq.data_ptr<float>(), stream());
}

void shard_adamw_allgather(torch::Tensor red, torch::Tensor master_local, torch::Tensor m,
                           torch::Tensor v, torch::Tensor master_table, torch::Tensor compute_table,
                           int64_t world, int64_t off, int64_t len, int64_t decay_end,
                           c10::optional<torch::Tensor> norm_payloads, double max_norm, double lr,
                           double b1, double b2, double eps, double wd, double bc1, double bc2,
                           double grad_scale, int64_t rank, int64_t local_end) {
  for (auto* t : {&red, &m, &v})
    TORCH_CHECK(t->scalar_type() == torch::kFloat32 && t->numel() >= len && t->is_contiguous(), "shard buffers");
  TORCH_CHECK(master_local.scalar_type() == torch::kFloat32 && master_local.numel() >= off + len, "master");
  TORCH_CHECK(master_table.numel() == world && compute_table.numel() == world, "peer tables");
  const c10::cuda::CUDAGuard guard(red.device());
  ddb::ShardAdamWArgs a;
  a.red = red.data_ptr<float>(); a.master_local = master_local.data_ptr<float>();
  a.m = m.data_ptr<float>(); a.v = v.data_ptr<float>();
  a.peer_master = reinterpret_cast<float* const*>(master_table.data_ptr<int64_t>());
  a.peer_compute = reinterpret_cast<__nv_bfloat16* const*>(compute_table.data_ptr<int64_t>());
  a.world = world; a.off = off; a.len = len; a.decay_end = decay_end;
  if (norm_payloads) a.norm_payloads = norm_payloads->data_ptr<float>();
  a.max_norm = max_norm; a.lr = lr; a.b1 = b1; a.b2 = b2; a.eps = eps; a.wd = wd;
  a.bc1 = bc1; a.bc2 = bc2; a.grad_scale = grad_scale;
  a.rank = static_cast<int>(rank); a.local_end = local_end;
  ddb::shard_adamw_allgather(a, stream());
}

// ------------------------------------------------------------------ MoE
// mode 1: D[rows] = A[rows] B[e]^T per expert row-tile (A: [rows, K]; B: [E, N, K] or, b_t,
//         [E, K, N]); mode 2: D[e] (+)= A[seg e]^T B[seg e] (A: [rows, M], B: [rows, N]).
void gemm_grouped(torch::Tensor A, torch::Tensor B, torch::Tensor D, int64_t epi, bool b_t,
                  int64_t mode, torch::Tensor tile_expert, torch::Tensor tile_row,
                  torch::Tensor total_mtiles, torch::Tensor kstart, torch::Tensor kend,
                  int64_t max_mtiles, c10::optional<torch::Tensor> C,
                  c10::optional<torch::Tensor> D2) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_rows(A, "A");
  check_rows(D, "D");
  for (auto* t : {&tile_expert, &tile_row, &total_mtiles, &kstart, &kend})
    TORCH_CHECK(t->scalar_type() == torch::kInt32 && t->is_cuda(), "grouped tables must be int32 CUDA");
  const c10::cuda::CUDAGuard guard(A.device());
  ddb::GemmArgs a;
  a.grouped = mode;
  a.grp_tile_expert = tile_expert.data_ptr<int>();
  a.grp_tile_row = tile_row.data_ptr<int>();
  a.grp_total_mtiles = total_mtiles.data_ptr<int>();
  a.grp_kstart = kstart.data_ptr<int>();
  a.grp_kend = kend.data_ptr<int>();
  a.grp_max_mtiles = max_mtiles;
  if (mode == 1) {
    TORCH_CHECK(B.dim() == 3 && B.stride(2) == 1, "grouped mode 1: B [E, rows, cols]");
    a.a_mn_major = false;
    a.b_mn_major = b_t;
    a.M = A.size(0);
    a.K = A.size(1);
    a.N = b_t ? B.size(2) : B.size(1);
    TORCH_CHECK((b_t ? B.size(1) : B.size(2)) == a.K, "grouped: inner dimensions differ");
    a.batch = B.size(0);
    a.stride_b = B.stride(0);
    a.ldb = B.stride(1);
  } else {
    TORCH_CHECK(mode == 2 && B.dim() == 2, "grouped mode 2: B [rows, N]");
    check_rows(B, "B");
    a.a_mn_major = true;
    a.b_mn_major = true;
    a.M = A.size(1);
    a.K = A.size(0);
    a.N = B.size(1);
    TORCH_CHECK(B.size(0) == a.K, "grouped mode 2: A and B rows differ");
    a.batch = kstart.numel();
    a.ldb = B.stride(0);
    TORCH_CHECK(D.size(0) == static_cast<int64_t>(a.batch) * a.M, "grouped mode 2: D rows");
  }
  a.A = A.data_ptr(); a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.D = D.data_ptr(); a.ldd = D.stride(0);
  if (C) {
    check_bf16(*C, "C");
    check_rows(*C, "C");
    a.C = C->data_ptr(); a.ldc = C->stride(0);
  }
  if (D2) {
    check_bf16(*D2, "D2");
    check_rows(*D2, "D2");
    a.D2 = D2->data_ptr(); a.ldd2 = D2->stride(0);
  }
  ddb::gemm(a, static_cast<int>(epi), stream());
}

std::vector<torch::Tensor> moe_route(torch::Tensor logits, c10::optional<torch::Tensor> bias,
                                     int64_t E, int64_t k, int64_t ns, bool want_probs) {
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.dim() == 2 && logits.stride(1) == 1,
              "logits must be fp32 [N, cols]");
  TORCH_CHECK(logits.size(1) >= E + ns, "logits too narrow");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0);
  auto opt = logits.options();
  auto idx = torch::empty({N, k}, opt.dtype(torch::kInt32));
  auto w = torch::empty({N, k}, opt);
  auto sw = torch::empty({N, std::max<int64_t>(ns, 1)}, opt);
  auto probs = want_probs ? torch::empty({N, E}, opt) : torch::empty({0}, opt);
  auto counts = torch::zeros({E}, opt.dtype(torch::kInt32));
  auto psum = torch::zeros({E}, opt);
  ddb::MoeRouteArgs a;
  a.logits = logits.data_ptr<float>(); a.ld_logits = logits.stride(0);
  if (bias) a.bias = bias->data_ptr<float>();
  a.N = N; a.E = E; a.k = k; a.ns = ns;
  a.topk_idx = idx.data_ptr<int>(); a.topk_w = w.data_ptr<float>(); a.shared_w = sw.data_ptr<float>();
  a.probs = want_probs ? probs.data_ptr<float>() : nullptr;
  a.counts = counts.data_ptr<int>(); a.psum = psum.data_ptr<float>();
  ddb::moe_route(a, stream());
  return {idx, w, sw, probs, counts, psum};
}

std::vector<torch::Tensor> moe_plan(torch::Tensor counts, int64_t E, int64_t ns, int64_t N,
                                    int64_t max_mtiles) {
  const c10::cuda::CUDAGuard guard(counts.device());
  auto opt = counts.options().dtype(torch::kInt32);
  const int64_t Ep = E + ns;
  auto seg_start = torch::empty({Ep}, opt), seg_count = torch::empty({Ep}, opt);
  auto tile_expert = torch::empty({max_mtiles}, opt), tile_row = torch::empty({max_mtiles}, opt);
  auto total = torch::empty({1}, opt), kstart = torch::empty({Ep}, opt), kend = torch::empty({Ep}, opt);
  auto cursor = torch::empty({Ep}, opt);
  ddb::moe_plan(counts.data_ptr<int>(), E, ns, N, seg_start.data_ptr<int>(), seg_count.data_ptr<int>(),
                tile_expert.data_ptr<int>(), tile_row.data_ptr<int>(), total.data_ptr<int>(),
                kstart.data_ptr<int>(), kend.data_ptr<int>(), cursor.data_ptr<int>(), max_mtiles,
                stream());
  return {seg_start, seg_count, tile_expert, tile_row, total, kstart, kend, cursor};
}

torch::Tensor moe_dispatch(torch::Tensor x, torch::Tensor topk_idx, torch::Tensor seg_start,
                           torch::Tensor seg_count, torch::Tensor cursor, torch::Tensor xp,
                           int64_t E, int64_t ns, c10::optional<torch::Tensor> xp2,
                           bool zero_routed_pad) {
  check_bf16(x, "x");
  check_bf16(xp, "xp");
  check_rows(x, "x");
  check_rows(xp, "xp");
  __nv_bfloat16* p2 = nullptr;
  int64_t ld2 = 0;
  if (xp2) {
    check_bf16(*xp2, "xp2");
    check_rows(*xp2, "xp2");
    p2 = reinterpret_cast<__nv_bfloat16*>(xp2->data_ptr());
    ld2 = xp2->stride(0);
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), k = topk_idx.size(1);
  auto slot_of = torch::empty({N, k + ns}, x.options().dtype(torch::kInt32));
  ddb::moe_dispatch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), N, x.size(1), k,
                    ns, E, topk_idx.data_ptr<int>(), seg_start.data_ptr<int>(), seg_count.data_ptr<int>(),
                    cursor.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(xp.data_ptr()),
                    xp.stride(0), slot_of.data_ptr<int>(), stream(), p2, ld2, zero_routed_pad,
                    xp.size(0), xp2 ? xp2->size(0) : 0);
  return slot_of;
}

void moe_zero_pad(torch::Tensor seg_start, torch::Tensor seg_count, torch::Tensor xp) {
  check_bf16(xp, "xp");
  check_rows(xp, "xp");
  TORCH_CHECK(seg_start.scalar_type() == torch::kInt32 && seg_count.scalar_type() == torch::kInt32 &&
                  seg_start.is_cuda() && seg_count.numel() == seg_start.numel(), "segment tables");
  const c10::cuda::CUDAGuard guard(xp.device());
  ddb::moe_zero_pad(seg_start.data_ptr<int>(), seg_count.data_ptr<int>(), seg_start.numel(),
                    reinterpret_cast<__nv_bfloat16*>(xp.data_ptr()), xp.stride(0), xp.size(1), stream());
}

ddb::MoeCombineArgs combine_args(torch::Tensor topk_w, torch::Tensor shared_w, torch::Tensor slot_of,
                                 torch::Tensor y, int64_t ns, const c10::optional<torch::Tensor>& y2) {
  check_bf16(y, "y");
  check_rows(y, "y");
  ddb::MoeCombineArgs a;
  a.N = topk_w.size(0); a.k = topk_w.size(1); a.ns = ns; a.d = y.size(1);
  a.topk_w = topk_w.data_ptr<float>(); a.shared_w = shared_w.data_ptr<float>();
  a.slot_of = slot_of.data_ptr<int>();
  a.y = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()); a.ld_y = y.stride(0);
  a.y_rows = y.size(0);
  if (y2) {
    check_bf16(*y2, "y2");
    check_rows(*y2, "y2");
    TORCH_CHECK(y2->size(1) == y.size(1), "y2 width");
    a.y2 = reinterpret_cast<const __nv_bfloat16*>(y2->data_ptr());
    a.ld_y2 = y2->stride(0);
    a.y2_rows = y2->size(0);
  }
  return a;
}

torch::Tensor moe_combine(torch::Tensor topk_w, torch::Tensor shared_w, torch::Tensor slot_of,
                          torch::Tensor y, c10::optional<torch::Tensor> residual, int64_t ns,
                          c10::optional<torch::Tensor> y2) {
  const c10::cuda::CUDAGuard guard(y.device());
  auto a = combine_args(topk_w, shared_w, slot_of, y, ns, y2);
  auto out = torch::empty({a.N, a.d}, y.options());
  if (residual) {
    check_bf16(*residual, "residual");
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ld_res = residual->stride(0);
  }
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr()); a.ld_out = out.stride(0);
  ddb::moe_combine(a, stream());
  return out;
}

// dy (and dy2 for the shared rows when y2 is given) may be supplied as outputs; rows no
// route writes keep their contents (a fresh dy is zero-filled).
std::vector<torch::Tensor> moe_combine_bwd(torch::Tensor topk_w, torch::Tensor shared_w,
                                           torch::Tensor slot_of, torch::Tensor y, torch::Tensor dout,
                                           int64_t ns, c10::optional<torch::Tensor> y2,
                                           c10::optional<torch::Tensor> dy_out,
                                           c10::optional<torch::Tensor> dy2_out) {
  const c10::cuda::CUDAGuard guard(y.device());
  auto a = combine_args(topk_w, shared_w, slot_of, y, ns, y2);
  check_bf16(dout, "dout");
  torch::Tensor dy = dy_out ? *dy_out : torch::zeros_like(y);
  check_bf16(dy, "dy");
  TORCH_CHECK(dy.stride(0) == a.ld_y && dy.size(0) >= y.size(0), "dy must match y's layout");
  torch::Tensor dy2;
  if (y2) {
    dy2 = dy2_out ? *dy2_out : torch::zeros_like(*y2);
    check_bf16(dy2, "dy2");
    TORCH_CHECK(dy2.stride(0) == a.ld_y2 && dy2.size(0) >= y2->size(0), "dy2 must match y2's layout");
  }
  auto dw = torch::empty({a.N, a.k + ns}, topk_w.options());
  ddb::moe_combine_bwd(a, reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
                       reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()), dw.data_ptr<float>(), stream(),
                       y2 ? reinterpret_cast<__nv_bfloat16*>(dy2.data_ptr()) : nullptr);
  if (y2) return {dy, dw, dy2};
  return {dy, dw};
}

torch::Tensor moe_unpermute(torch::Tensor dxp, torch::Tensor slot_of, int64_t N,
                            c10::optional<torch::Tensor> dxp2, int64_t k) {
  check_bf16(dxp, "dxp");
  const __nv_bfloat16* p2 = nullptr;
  int64_t ld2 = 0;
  if (dxp2) {
    check_bf16(*dxp2, "dxp2");
    TORCH_CHECK(dxp2->size(1) == dxp.size(1), "dxp2 width");
    p2 = reinterpret_cast<const __nv_bfloat16*>(dxp2->data_ptr());
    ld2 = dxp2->stride(0);
  }
  const c10::cuda::CUDAGuard guard(dxp.device());
  auto dx = torch::empty({N, dxp.size(1)}, dxp.options());
  ddb::moe_unpermute(reinterpret_cast<const __nv_bfloat16*>(dxp.data_ptr()), dxp.stride(0),
                     slot_of.data_ptr<int>(), N, slot_of.size(1), dxp.size(1),
                     reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dx.stride(0), stream(), k, p2, ld2,
                     dxp.size(0), dxp2 ? dxp2->size(0) : 0);
  return dx;
}

// ---------------------------------------------------------------- video VAE
void check_cl5(const torch::Tensor& t, const char* name) {
  check_bf16(t, name);
  TORCH_CHECK(t.dim() == 5 && t.is_contiguous(), name, " must be a contiguous [B,T,H,W,C] tensor");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

// y[B,To,Ho,Wo,Cout] = conv(x[B,T,H,W,Cin], w[Cout, kt*kh*kw*Cin]) (+bias) (+residual)
void conv3d_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y, int64_t kt, int64_t kh,
                int64_t kw, int64_t pt, int64_t ph, int64_t pw,
                c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> residual) {
  check_cl5(x, "x");
  check_cl5(y, "y");
  check_bf16(w, "w");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous(), "w must be contiguous [Cout, K]");
  const int64_t Cin = x.size(4), Cout = y.size(4);
  TORCH_CHECK(w.size(0) == Cout && w.size(1) == kt * kh * kw * Cin, "w shape");
  TORCH_CHECK(y.size(0) == x.size(0), "batch");
  const c10::cuda::CUDAGuard guard(x.device());
  ddb::Conv3dArgs a;
  a.x = x.data_ptr(); a.B = x.size(0); a.T = x.size(1); a.H = x.size(2); a.W = x.size(3);
  a.Cin = Cin; a.To = y.size(1); a.Ho = y.size(2); a.Wo = y.size(3); a.Cout = Cout;
  a.kt = kt; a.kh = kh; a.kw = kw; a.pt = pt; a.ph = ph; a.pw = pw;
  a.w = w.data_ptr(); a.y = y.data_ptr();
  if (bias) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() == Cout &&
                bias->is_contiguous(), "bias must be fp32 [Cout]");
    a.bias = bias->data_ptr<float>();
  }
  if (residual) {
    check_cl5(*residual, "residual");
    TORCH_CHECK(residual->sizes() == y.sizes(), "residual shape");
    a.residual = residual->data_ptr();
  }
  ddb::conv3d_fwd(a, stream());
}

// dw[Cout, kt*kh*kw*Cin] (fp32) += weight gradient of conv(x) given dy
void conv3d_wgrad(torch::Tensor x, torch::Tensor dy, torch::Tensor dw, int64_t kt, int64_t kh,
                  int64_t kw, int64_t pt, int64_t ph, int64_t pw, int64_t splits) {
  check_cl5(x, "x");
  check_cl5(dy, "dy");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.is_contiguous() && dw.dim() == 2,
              "dw must be contiguous fp32 [Cout, K]");
  const int64_t Cin = x.size(4), Cout = dy.size(4);
  TORCH_CHECK(dw.size(0) == Cout && dw.size(1) == kt * kh * kw * Cin, "dw shape");
  const c10::cuda::CUDAGuard guard(x.device());
  ddb::Conv3dArgs a;
  a.x = x.data_ptr(); a.B = x.size(0); a.T = x.size(1); a.H = x.size(2); a.W = x.size(3);
  a.Cin = Cin; a.To = dy.size(1); a.Ho = dy.size(2); a.Wo = dy.size(3); a.Cout = Cout;
  a.kt = kt; a.kh = kh; a.kw = kw; a.pt = pt; a.ph = ph; a.pw = pw;
  a.dy = dy.data_ptr(); a.dw = dw.data_ptr<float>(); a.splits = splits;
  ddb::conv3d_wgrad(a, stream());
}

// GroupNorm(+SiLU) over x[B, P, C] -> (y, stats[B,G,2])
std::vector<torch::Tensor> groupnorm_fwd(torch::Tensor x, torch::Tensor w,
                                         c10::optional<torch::Tensor> b, int64_t G, double eps,
                                         bool silu) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous(), "x must be contiguous [B, P, C]");
  const int64_t B = x.size(0), P = x.size(1), C = x.size(2);
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.numel() == C && w.is_contiguous(), "w");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto stats = torch::empty({B, G, 2}, x.options().dtype(torch::kFloat32));
  auto acc = torch::empty({B, C, 2}, x.options().dtype(torch::kFloat64));
  ddb::GroupNormArgs a;
  a.B = B; a.P = P; a.C = C; a.G = G; a.eps = static_cast<float>(eps); a.silu = silu;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()); a.w = w.data_ptr<float>();
  if (b) {
    TORCH_CHECK(b->scalar_type() == torch::kFloat32 && b->numel() == C && b->is_contiguous(), "b");
    a.b = b->data_ptr<float>();
  }
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.stats = stats.data_ptr<float>(); a.acc = acc.data_ptr<double>();
  ddb::groupnorm_fwd(a, stream());
  return {y, stats};
}

// -> (dx, per-sample channel sums [B, C, 2] = (sum dpre, sum dpre*xhat)) in fp64
std::vector<torch::Tensor> groupnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                         c10::optional<torch::Tensor> b, torch::Tensor stats,
                                         bool silu) {
  check_bf16(x, "x");
  check_bf16(dy, "dy");
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous() && dy.is_contiguous() && dy.sizes() == x.sizes(),
              "x/dy must be contiguous [B, P, C]");
  const int64_t B = x.size(0), P = x.size(1), C = x.size(2), G = stats.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  auto acc = torch::empty({B, C, 2}, x.options().dtype(torch::kFloat64));
  auto coef = torch::empty({B, G, 2}, x.options().dtype(torch::kFloat32));
  ddb::GroupNormArgs a;
  a.B = B; a.P = P; a.C = C; a.G = G; a.silu = silu;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()); a.w = w.data_ptr<float>();
  if (b) a.b = b->data_ptr<float>();
  a.stats = stats.data_ptr<float>(); a.acc = acc.data_ptr<double>(); a.coef = coef.data_ptr<float>();
  a.dy = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  a.dx = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  ddb::groupnorm_bwd(a, stream());
  return {dx, acc};
}


// LayerNorm over rows: -> (y, mean, rstd)
std::vector<torch::Tensor> layernorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> w,
                                         c10::optional<torch::Tensor> b, double eps) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "x must be contiguous [M, D]");
  const int64_t M = x.size(0), D = x.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto mean = torch::empty({M}, x.options().dtype(torch::kFloat32));
  auto rstd = torch::empty({M}, x.options().dtype(torch::kFloat32));
  ddb::LayerNormArgs a;
  a.M = M; a.D = D; a.eps = static_cast<float>(eps);
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  if (w) {
    TORCH_CHECK(w->scalar_type() == torch::kFloat32 && w->numel() == D && w->is_contiguous(), "w");
    a.w = w->data_ptr<float>();
  }
  if (b) {
    TORCH_CHECK(b->scalar_type() == torch::kFloat32 && b->numel() == D && b->is_contiguous(), "b");
    a.b = b->data_ptr<float>();
  }
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.mean = mean.data_ptr<float>(); a.rstd = rstd.data_ptr<float>();
  ddb::layernorm_fwd(a, stream());
  return {y, mean, rstd};
}

// -> dx; accumulates dw / db (fp32, optional)
torch::Tensor layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor mean,
                            torch::Tensor rstd, c10::optional<torch::Tensor> w,
                            c10::optional<torch::Tensor> dw, c10::optional<torch::Tensor> db) {
  check_bf16(dy, "dy");
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && dy.is_contiguous() && dy.sizes() == x.sizes(),
              "x / dy must be contiguous [M, D]");
  const int64_t M = x.size(0), D = x.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  ddb::LayerNormArgs a;
  a.M = M; a.D = D;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.dy = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  a.dx = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  a.mean = mean.data_ptr<float>(); a.rstd = rstd.data_ptr<float>();
  if (w) a.w = w->data_ptr<float>();
  if (dw) {
    TORCH_CHECK(dw->scalar_type() == torch::kFloat32 && dw->numel() == D && dw->is_contiguous(), "dw");
    a.dw = dw->data_ptr<float>();
  }
  if (db) {
    TORCH_CHECK(db->scalar_type() == torch::kFloat32 && db->numel() == D && db->is_contiguous(), "db");
    a.db = db->data_ptr<float>();
  }
  ddb::layernorm_bwd(a, stream());
  return dx;
}


// fused flip / brightness / contrast / normalise (+ HWC uint8 -> CHW) over a clip batch
torch::Tensor video_augment(torch::Tensor x, bool input_u8_hwc, bool out_bf16,
                            c10::optional<torch::Tensor> flip, c10::optional<torch::Tensor> brightness,
                            c10::optional<torch::Tensor> contrast, c10::optional<torch::Tensor> mean,
                            c10::optional<torch::Tensor> std_) {
  check_cuda_tensor(x, "x");
  TORCH_CHECK(x.dim() == 5 && x.is_contiguous(), "x must be a contiguous 5-D clip batch");
  if (input_u8_hwc) {
    TORCH_CHECK(x.scalar_type() == torch::kUInt8, "uint8 HWC input expected");
  } else {
    TORCH_CHECK(x.scalar_type() == torch::kFloat32, "float32 CHW input expected");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  ddb::AugmentArgs a;
  a.B = x.size(0); a.T = x.size(1);
  if (input_u8_hwc) { a.H = x.size(2); a.W = x.size(3); a.C = x.size(4); }
  else { a.C = x.size(2); a.H = x.size(3); a.W = x.size(4); }
  a.x = x.data_ptr(); a.input_u8_hwc = input_u8_hwc; a.out_bf16 = out_bf16;
  auto y = torch::empty({a.B, a.T, a.C, a.H, a.W},
                        x.options().dtype(out_bf16 ? torch::kBFloat16 : torch::kFloat32));
  a.y = y.data_ptr();
  auto f32 = [&](const c10::optional<torch::Tensor>& t, int64_t n, const char* nm) -> const float* {
    if (!t) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->numel() == n && t->is_contiguous(), nm);
    return t->data_ptr<float>();
  };
  if (flip) {
    TORCH_CHECK(flip->is_cuda() && flip->scalar_type() == torch::kInt32 && flip->numel() == a.B, "flip");
    a.flip = flip->data_ptr<int>();
  }
  a.brightness = f32(brightness, a.B, "brightness");
  a.contrast = f32(contrast, a.B, "contrast");
  a.mean = f32(mean, a.C, "mean");
  a.std = f32(std_, a.C, "std");
  TORCH_CHECK((a.mean == nullptr) == (a.std == nullptr), "mean and std go together");
  ddb::video_augment(a, stream());
  return y;
}


// Owner-driven expert parallelism. Tables are int64 device arrays of per-rank base
// pointers (routing ids, routing weights, rows, return / dw buffers).
ddb::EpOwnerArgs ep_owner_args(torch::Tensor peer_idx, torch::Tensor peer_w, torch::Tensor peer_rows,
                               int64_t world, int64_t rank, int64_t N, int64_t k, int64_t d, int64_t lo,
                               int64_t El, torch::Tensor seg_start, torch::Tensor cursor,
                               torch::Tensor meta, torch::Tensor meta_w, torch::Tensor n_uniq) {
  for (auto* t : {&peer_idx, &peer_w, &peer_rows})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt64 && t->numel() == world, "peer tables");
  for (auto* t : {&seg_start, &cursor, &meta, &n_uniq})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->is_contiguous(), "int32 EP state");
  TORCH_CHECK(meta_w.scalar_type() == torch::kFloat32 && meta_w.is_contiguous(), "meta_w");
  TORCH_CHECK(meta.dim() == 2 && meta.size(1) == 2 + k && meta_w.size(0) == meta.size(0), "meta shape");
  ddb::EpOwnerArgs a;
  a.world = world; a.rank = rank; a.N = N; a.k = k; a.d = d; a.lo = lo; a.El = El;
  a.peer_idx = reinterpret_cast<const int* const*>(peer_idx.data_ptr<int64_t>());
  a.peer_w = reinterpret_cast<const float* const*>(peer_w.data_ptr<int64_t>());
  a.peer_rows = reinterpret_cast<const __nv_bfloat16* const*>(peer_rows.data_ptr<int64_t>());
  a.seg_start = seg_start.data_ptr<int>();
  a.cursor = cursor.data_ptr<int>();
  a.meta = meta.data_ptr<int>();
  a.meta_w = meta_w.data_ptr<float>();
  a.n_uniq = n_uniq.data_ptr<int>();
  a.cap = meta.size(0);
  return a;
}

// Source push of token rows (h, or dout in gradient mode) into the owners' staging rows.
void ep_push_rows(torch::Tensor idx, c10::optional<torch::Tensor> w, torch::Tensor rows,
                  torch::Tensor stage_table, c10::optional<torch::Tensor> smeta_table,
                  c10::optional<torch::Tensor> cnt, torch::Tensor pos, int64_t world, int64_t rank,
                  int64_t El) {
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == torch::kInt32 && idx.dim() == 2 && idx.is_contiguous(), "idx");
  check_bf16(rows, "rows");
  check_rows(rows, "rows");
  const int64_t N = idx.size(0), k = idx.size(1);
  TORCH_CHECK(rows.size(0) == N, "rows / idx");
  TORCH_CHECK(stage_table.scalar_type() == torch::kInt64 && stage_table.numel() == world, "stage table");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && pos.is_contiguous() && pos.numel() == N * world, "pos [N, world]");
  const c10::cuda::CUDAGuard guard(rows.device());
  ddb::EpPushArgs a;
  a.world = world; a.rank = rank; a.N = N; a.k = k; a.d = rows.size(1); a.El = El;
  a.idx = idx.data_ptr<int>();
  a.rows = reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr());
  a.ld_rows = rows.stride(0);
  a.stage = reinterpret_cast<__nv_bfloat16* const*>(stage_table.data_ptr<int64_t>());
  a.pos = pos.data_ptr<int>();
  if (smeta_table) {
    TORCH_CHECK(w && cnt, "forward push needs weights and the owner counters");
    TORCH_CHECK(w->scalar_type() == torch::kFloat32 && w->is_contiguous() && w->numel() == N * k, "w");
    TORCH_CHECK(cnt->scalar_type() == torch::kInt32 && cnt->numel() == world, "cnt");
    TORCH_CHECK(smeta_table->scalar_type() == torch::kInt64 && smeta_table->numel() == world, "smeta table");
    a.w = w->data_ptr<float>();
    a.cnt = cnt->data_ptr<int>();
    a.smeta = reinterpret_cast<int* const*>(smeta_table->data_ptr<int64_t>());
  }
  ddb::ep_push_rows(a, stream());
}

// Owner fan-out of the staged rows into the local expert segments.
void ep_owner_fanout(int64_t stage_ptr, int64_t smeta_ptr, torch::Tensor prefix, int64_t total, int64_t world,
                     int64_t N, int64_t k, int64_t d, int64_t lo, int64_t El, torch::Tensor seg_start,
                     torch::Tensor cursor, torch::Tensor xr, torch::Tensor meta, torch::Tensor meta_w,
                     torch::Tensor urow, torch::Tensor n_uniq) {
  check_bf16(xr, "xr");
  check_rows(xr, "xr");
  TORCH_CHECK(xr.size(1) == d, "xr width");
  for (auto* t : {&prefix, &seg_start, &cursor, &meta, &urow, &n_uniq})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->is_contiguous(), "int32 EP state");
  TORCH_CHECK(prefix.numel() == world + 1, "prefix [world + 1]");
  TORCH_CHECK(meta.dim() == 2 && meta.size(1) == 2 + k && meta.size(0) >= total && meta_w.size(0) >= total &&
                  urow.numel() >= total, "meta capacity");
  const c10::cuda::CUDAGuard guard(xr.device());
  ddb::EpFanoutArgs a;
  a.world = world; a.N = N; a.k = k; a.d = d; a.lo = lo; a.El = El; a.total = total;
  a.stage = reinterpret_cast<const __nv_bfloat16*>(stage_ptr);
  a.smeta = reinterpret_cast<const int*>(smeta_ptr);
  a.prefix = prefix.data_ptr<int>();
  a.seg_start = seg_start.data_ptr<int>();
  a.cursor = cursor.data_ptr<int>();
  a.xr = reinterpret_cast<__nv_bfloat16*>(xr.data_ptr());
  a.ld_xr = xr.stride(0);
  a.meta = meta.data_ptr<int>();
  a.meta_w = meta_w.data_ptr<float>();
  a.urow = urow.data_ptr<int>();
  a.n_uniq = n_uniq.data_ptr<int>();
  ddb::ep_owner_fanout(a, stream());
}

void ep_owner_grad_gather(torch::Tensor peer_idx, torch::Tensor peer_w, torch::Tensor peer_rows,
                          int64_t world, int64_t rank, int64_t N, int64_t k, int64_t d, int64_t lo, int64_t El,
                          torch::Tensor seg_start, torch::Tensor cursor, torch::Tensor meta,
                          torch::Tensor meta_w, torch::Tensor n_uniq, torch::Tensor y, torch::Tensor dy,
                          torch::Tensor peer_dw, int64_t local_rows, c10::optional<torch::Tensor> urow) {
  check_bf16(y, "y");
  check_bf16(dy, "dy");
  check_rows(y, "y");
  check_rows(dy, "dy");
  TORCH_CHECK(peer_dw.scalar_type() == torch::kInt64 && peer_dw.numel() == world, "dw table");
  const c10::cuda::CUDAGuard guard(y.device());
  auto a = ep_owner_args(peer_idx, peer_w, peer_rows, world, rank, N, k, d, lo, El, seg_start, cursor, meta,
                         meta_w, n_uniq);
  if (local_rows != 0) {  // dout rows pushed into this rank's staging buffer
    TORCH_CHECK(urow && urow->scalar_type() == torch::kInt32 && urow->numel() >= meta.size(0), "urow");
    a.local_rows = reinterpret_cast<const __nv_bfloat16*>(local_rows);
    a.urow = urow->data_ptr<int>();
  }
  ddb::ep_owner_grad_gather(a, reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0),
                            reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()), dy.stride(0),
                            reinterpret_cast<float* const*>(peer_dw.data_ptr<int64_t>()), stream());
}

void ep_owner_scatter_sum(torch::Tensor peer_idx, torch::Tensor peer_w, torch::Tensor peer_rows,
                          int64_t world, int64_t rank, int64_t N, int64_t k, int64_t d, int64_t lo, int64_t El,
                          torch::Tensor seg_start, torch::Tensor cursor, torch::Tensor meta,
                          torch::Tensor meta_w, torch::Tensor n_uniq, torch::Tensor src, bool weighted,
                          torch::Tensor peer_ret) {
  check_bf16(src, "src");
  check_rows(src, "src");
  TORCH_CHECK(peer_ret.scalar_type() == torch::kInt64 && peer_ret.numel() == world, "return table");
  const c10::cuda::CUDAGuard guard(src.device());
  auto a = ep_owner_args(peer_idx, peer_w, peer_rows, world, rank, N, k, d, lo, El, seg_start, cursor, meta,
                         meta_w, n_uniq);
  ddb::ep_owner_scatter_sum(a, reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.stride(0), weighted,
                            reinterpret_cast<__nv_bfloat16* const*>(peer_ret.data_ptr<int64_t>()), stream());
}

torch::Tensor ep_source_reduce(torch::Tensor idx, torch::Tensor ret, int64_t El,
                               c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> shared_w,
                               c10::optional<torch::Tensor> slot_s, c10::optional<torch::Tensor> ys) {
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.dim() == 2 && idx.is_contiguous(), "idx [N, k] int32");
  check_bf16(ret, "ret");
  TORCH_CHECK(ret.is_contiguous() && ret.dim() == 2, "ret [world * N, d] contiguous");
  const c10::cuda::CUDAGuard guard(ret.device());
  ddb::EpSourceArgs a;
  a.N = idx.size(0); a.k = idx.size(1); a.d = ret.size(1); a.El = El;
  a.idx = idx.data_ptr<int>();
  a.ret = reinterpret_cast<const __nv_bfloat16*>(ret.data_ptr());
  if (residual) {
    check_bf16(*residual, "residual");
    check_rows(*residual, "residual");
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ld_res = residual->stride(0);
  }
  if (slot_s) {
    TORCH_CHECK(ys.has_value(), "shared rows");
    TORCH_CHECK(slot_s->scalar_type() == torch::kInt32 && slot_s->is_contiguous(), "slot_s int32");
    check_bf16(*ys, "ys");
    check_rows(*ys, "ys");
    a.ns = slot_s->size(1);
    a.slot_s = slot_s->data_ptr<int>();
    a.ys = reinterpret_cast<const __nv_bfloat16*>(ys->data_ptr());
    a.ld_ys = ys->stride(0);
    if (shared_w) {
      TORCH_CHECK(shared_w->scalar_type() == torch::kFloat32 && shared_w->is_contiguous(), "shared_w");
      a.shared_w = shared_w->data_ptr<float>();
    }
  }
  auto out = torch::empty({a.N, a.d}, ret.options());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ld_out = out.stride(0);
  ddb::ep_source_reduce(a, stream());
  return out;
}

// Row-block copies for expert parallelism: blocks [n, 4] int32 (src_rank, src_row, dst_rank,
// dst_row), row_prefix [n] int32 (first flat row of each block). A side is either a table of
// per-rank base pointers (int64 device array) or one local base pointer.
void ep_copy_rows(c10::optional<torch::Tensor> src_table, int64_t src_ptr,
                  c10::optional<torch::Tensor> dst_table, int64_t dst_ptr, torch::Tensor blocks,
                  torch::Tensor row_prefix, int64_t total_rows, int64_t row_bytes, int64_t src_ld,
                  int64_t dst_ld) {
  for (auto* t : {&src_table, &dst_table})
    if (*t) TORCH_CHECK((*t)->is_cuda() && (*t)->scalar_type() == torch::kInt64 && (*t)->is_contiguous(),
                        "pointer tables must be int64 device arrays");
  TORCH_CHECK(src_table || src_ptr, "ep_copy_rows: no source");
  TORCH_CHECK(dst_table || dst_ptr, "ep_copy_rows: no destination");
  for (auto* t : {&blocks, &row_prefix})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->is_contiguous(), "int32 device block list");
  TORCH_CHECK(blocks.dim() == 2 && blocks.size(1) == 4 && row_prefix.numel() == blocks.size(0), "block list");
  const c10::cuda::CUDAGuard guard(blocks.device());
  ddb::EpCopyArgs a;
  if (src_table) a.src_table = reinterpret_cast<const void* const*>(src_table->data_ptr<int64_t>());
  if (dst_table) a.dst_table = reinterpret_cast<void* const*>(dst_table->data_ptr<int64_t>());
  a.src_local = reinterpret_cast<const void*>(src_ptr);
  a.dst_local = reinterpret_cast<void*>(dst_ptr);
  a.blocks = blocks.data_ptr<int>();
  a.row_prefix = row_prefix.data_ptr<int>();
  a.nblocks = blocks.size(0);
  a.total_rows = total_rows;
  a.row_bytes = row_bytes;
  a.src_ld = src_ld;
  a.dst_ld = dst_ld;
  ddb::ep_copy_rows(a, stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "drivedit_b200 sm_100a kernels";
  m.def("conv3d_fwd", &conv3d_fwd, "causal 3-D conv (channels-last implicit GEMM, tcgen05)");
  m.def("conv3d_wgrad", &conv3d_wgrad, "causal 3-D conv weight gradient (fp32 accumulate)");
  m.def("groupnorm_fwd", &groupnorm_fwd, "GroupNorm(+SiLU) forward -> (y, stats)");
  m.def("groupnorm_bwd", &groupnorm_bwd, "GroupNorm(+SiLU) backward -> (dx, channel sums)");
  m.def("layernorm_fwd", &layernorm_fwd, "LayerNorm forward -> (y, mean, rstd)");
  m.def("layernorm_bwd", &layernorm_bwd, "LayerNorm backward -> dx (accumulates dw, db)");
  m.def("video_augment", &video_augment, "fused flip/brightness/contrast/normalise of clips");
  m.def("ep_copy_rows", &ep_copy_rows, "row-block copies between local and peer buffers (EP)");
  m.def("ep_owner_grad_gather", &ep_owner_grad_gather, "EP backward dispatch: dy rows and routing-weight grads",
        py::arg("peer_idx"), py::arg("peer_w"), py::arg("peer_rows"), py::arg("world"), py::arg("rank"),
        py::arg("N"), py::arg("k"), py::arg("d"), py::arg("lo"), py::arg("El"), py::arg("seg_start"),
        py::arg("cursor"), py::arg("meta"), py::arg("meta_w"), py::arg("n_uniq"), py::arg("y"), py::arg("dy"),
        py::arg("peer_dw"), py::arg("local_rows") = 0, py::arg("urow") = py::none());
  m.def("ep_push_rows", &ep_push_rows, "EP dispatch: source pushes token rows to their owners' staging",
        py::arg("idx"), py::arg("w"), py::arg("rows"), py::arg("stage_table"), py::arg("smeta_table"),
        py::arg("cnt"), py::arg("pos"), py::arg("world"), py::arg("rank"), py::arg("El"));
  m.def("ep_owner_fanout", &ep_owner_fanout, "EP dispatch: owner fans staged rows out to expert segments");
  m.def("ep_owner_scatter_sum", &ep_owner_scatter_sum, "EP combine: owner-side partial sums pushed to sources");
  m.def("ep_source_reduce", &ep_source_reduce, "EP source-side sum of owner partials (+ shared, residual)",
        py::arg("idx"), py::arg("ret"), py::arg("El"), py::arg("residual") = py::none(),
        py::arg("shared_w") = py::none(), py::arg("slot_s") = py::none(), py::arg("ys") = py::none());
  m.def("gemm", &gemm, "tcgen05 GEMM D = A B^T with fused epilogue");
  m.def("gemm_set_pair_mode", [](int64_t mode) { return static_cast<int64_t>(ddb::gemm_set_pair_mode(static_cast<int>(mode))); },
        "CTA-pair GEMM tiles: -1 auto, 0 off, 1 whenever eligible; returns the previous mode");
  m.def("read_status", &read_status, "device status word (0 = ok)");
  m.def("read_status_index", &read_status_index, "index recorded with a bad-index status");
  m.def("set_deterministic", &ddb::set_deterministic, "fixed-order MoE permutation on/off");
  m.def("deterministic", &ddb::deterministic, "fixed-order MoE permutation enabled");
  m.def("set_check_bounds", &ddb::set_check_bounds, "bounds-checked index kernels on/off");
  m.def("check_bounds", &ddb::check_bounds, "bounds-checked index kernels enabled");
  m.def("launch_count", &ddb::launch_count, "kernels launched by this extension so far");
  m.def("reset_status", &reset_status, "clear the device status word");
  m.def("adaln_fwd", &adaln_fwd, "fused AdaLN-RMSNorm forward -> (h, rstd)");
  m.def("adaln_bwd", &adaln_bwd, "fused AdaLN-RMSNorm backward -> dx (accumulates dw, dmod)");
  m.def("adamw_flat", &adamw_flat, "flat AdamW + bf16 copy");
  m.def("cast_bf16", &cast_bf16, "fp32 -> bf16 cast");
  m.def("sq_norm", &sq_norm, "sum of squares (fp32)");
  m.def("rope_rotate", &rope_rotate, "in-place rotary rotation of leading columns");
  m.def("attn_fwd", &attn_fwd, "tcgen05 flash attention forward (dense / frame-causal / sparse)");
  m.def("attn_fwd_set_trace", &attn_fwd_set_trace, "clock64 trace of one forward CTA (None: off)");
  m.def("attn_fwd_set_kv_splits", [](int64_t n) { const int64_t prev = g_attn_kv_splits; g_attn_kv_splits = n < 0 ? 0 : n; return prev; },
        "split-KV of the attention forward: 0 = chosen per launch, n >= 1 = n splits; returns the previous setting");
  m.def("attn_bwd", &attn_bwd, "tcgen05 flash attention backward (KV-stationary)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("dout"), py::arg("lse"),
        py::arg("delta"), py::arg("dq_acc"), py::arg("dk"), py::arg("dv"), py::arg("q_col"),
        py::arg("k_col"), py::arg("v_col"), py::arg("o_col"), py::arg("do_col"), py::arg("dk_col"),
        py::arg("dv_col"), py::arg("B"), py::arg("H"), py::arg("Tq"), py::arg("S"),
        py::arg("q_rows_per_b"), py::arg("kv_rows_per_b"), py::arg("causal"), py::arg("tpf"),
        py::arg("q_pos_offset"), py::arg("kv_pos_offset"), py::arg("scale"), py::arg("kv_qtiles"),
        py::arg("kv_qmask"), py::arg("kv_count"), py::arg("debug_flags") = 0,
        py::arg("trace") = py::none(), py::arg("trace_cta") = 0);
  m.def("attn_delta", &attn_delta, "rowsum(dO * O) per head");
  m.def("ipc_alloc", &ipc_alloc, "cudaMalloc + IPC handle -> (ptr, handle)");
  m.def("ipc_open", &ipc_open, "open a peer's IPC handle -> ptr");
  m.def("ipc_close", &ipc_close, "close a peer mapping");
  m.def("ipc_free", &ipc_free, "free a local IPC buffer");
  m.def("tensor_from_ptr", &tensor_from_ptr, "tensor view of a device pointer");
  m.def("xrank_barrier", &xrank_barrier, "bounded cross-rank flag barrier over peer memory");
  m.def("gemm_tp", &gemm_tp, "tcgen05 GEMM with the all-gather of A and/or the reduce-scatter of D fused");
  m.def("tp_sum_rows", &tp_sum_rows, "sum of the per-rank partial rows (+ residual)");
  m.def("tp_allreduce_sum", &tp_allreduce_sum, "all-reduce by peer loads: residual + sum of every rank's partial");
  m.def("rs_sum_sqnorm", &rs_sum_sqnorm, "reduce-scatter by peer loads + squared norm");
  m.def("shard_adamw_allgather", &shard_adamw_allgather, "sharded AdamW + all-gather by peer stores");
  m.def("gemm_grouped", &gemm_grouped, "grouped (MoE) tcgen05 GEMM with device tile tables");
  m.def("moe_route", &moe_route, "MoE top-k routing (+ shared gates, counts, prob sums)");
  m.def("moe_plan", &moe_plan, "MoE segment layout and grouped-GEMM tables");
  m.def("moe_dispatch", &moe_dispatch, "MoE token permutation into expert segments",
        py::arg("x"), py::arg("topk_idx"), py::arg("seg_start"), py::arg("seg_count"), py::arg("cursor"),
        py::arg("xp"), py::arg("E"), py::arg("ns"), py::arg("xp2") = py::none(),
        py::arg("zero_routed_pad") = true);
  m.def("moe_zero_pad", &moe_zero_pad, "zero the padding rows of 128-row expert segments");
  m.def("moe_combine", &moe_combine, "MoE weighted combine (+ residual)", py::arg("topk_w"),
        py::arg("shared_w"), py::arg("slot_of"), py::arg("y"), py::arg("residual"), py::arg("ns"),
        py::arg("y2") = py::none());
  m.def("moe_combine_bwd", &moe_combine_bwd, "MoE combine backward", py::arg("topk_w"),
        py::arg("shared_w"), py::arg("slot_of"), py::arg("y"), py::arg("dout"), py::arg("ns"),
        py::arg("y2") = py::none(), py::arg("dy") = py::none(), py::arg("dy2") = py::none());
  m.def("moe_unpermute", &moe_unpermute, "MoE gather-sum of permuted gradients", py::arg("dxp"),
        py::arg("slot_of"), py::arg("N"), py::arg("dxp2") = py::none(), py::arg("k") = 0);
  m.def("gemm_batched", &gemm_batched, "strided-batched tcgen05 GEMM");
  m.def("sla_pool", &sla_pool, "SLA block means of q, k");
  m.def("sla_route", &sla_route, "SLA top-k routing + kernel lists");
  m.def("sla_kv_state", &sla_kv_state, "SLA per-block linear states");
  m.def("sla_lin_out", &sla_lin_out, "SLA linear-branch output");
  m.def("sla_lin_bwd_q", &sla_lin_bwd_q, "SLA linear-branch backward (query side)");
  m.def("sla_lin_bwd_kv", &sla_lin_bwd_kv, "SLA linear-branch backward (key side)");
  m.def("attn_dq_finalize", &attn_dq_finalize, "fp32 dq accumulator -> bf16 (+ inverse rope)");
}
