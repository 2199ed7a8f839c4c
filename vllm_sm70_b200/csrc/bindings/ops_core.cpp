// torch.ops._b200_C: the op registry of the B200 kernel library.
//
// Reference parity: TORCH_LIBRARY(_sm70_C) + abi_version
// (sm70/csrc/torch_bindings_sm70.cpp:16-40). Each area adds a FRAGMENT; this
// file holds the core ops (GEMM, norm, RoPE/KV, attention, sampling, misc).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>
#include <torch/torch.h>

#include "ops_api.h"
#include "comm/comm_api.h"
#include "moe/moe_api.h"
#include "sampler/sampler_api.h"
#include "gdn/gdn_api.h"

namespace b200 {
namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")
#define CHECK_ROWMAJOR(x) \
  TORCH_CHECK((x).dim() == 2 && (x).stride(1) == 1, #x " must be 2-D with unit inner stride")

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

int64_t abi_version() { return kAbiVersion; }

// cfg < 0: auto plan (tile + split-K). splits > 0 forces the split factor
// (used by tests); the split path needs the configured per-device workspace.
void launch_gemm(at::Tensor& out, const at::Tensor& a, const at::Tensor& w, int epi, int64_t cfg,
                 int64_t splits) {
  const int dev = a.get_device();
  const int M = (int)a.size(0), N = (int)w.size(0), K = (int)a.size(1);
  int c = (int)cfg, s = (int)splits;
  if (c < 0) {
    int nsm = 0;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    GemmPlan p = gemm_bf16_plan(M, N, K, epi, nsm);
    c = p.cfg;
    if (s <= 0) s = p.splits;
  }
  if (s <= 0) s = 1;
  gemm_bf16_launch_split(a.data_ptr(), w.data_ptr(), out.data_ptr(), M, N, K, (int)a.stride(0),
                         (int)w.stride(0), (int)out.stride(0), epi, c, s, gemm_ws_ptr(dev),
                         gemm_workspace_bytes(dev), gemm_counters_ptr(dev),
                         gemm_n_counters(dev), device_status_ptr(dev), cur_stream(),
                         /*ext_reduce=*/epi == kEpiNone);
}

void init_device(int64_t device) { (void)device_status_ptr((int)device); }

int64_t read_status(int64_t device, bool clear) {
  unsigned int* p = device_status_ptr((int)device);
  unsigned int v = 0;
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost));
  if (clear && v) C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(v)));
  return (int64_t)v;
}

void gemm_bf16_out(at::Tensor& out, const at::Tensor& a, const at::Tensor& w, int64_t cfg,
                   int64_t splits) {
  CHECK_CUDA(a); CHECK_CUDA(w); CHECK_CUDA(out);
  CHECK_BF16(a); CHECK_BF16(w); CHECK_BF16(out);
  CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(w); CHECK_ROWMAJOR(out);
  TORCH_CHECK(a.size(1) == w.size(1), "gemm_bf16: K mismatch");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == w.size(0), "gemm_bf16: out shape");
  c10::cuda::CUDAGuard g(a.device());
  launch_gemm(out, a, w, kEpiNone, cfg, splits);
}

at::Tensor gemm_bf16(const at::Tensor& a, const at::Tensor& w, int64_t cfg) {
  auto out = at::empty({a.size(0), w.size(0)}, a.options());
  gemm_bf16_out(out, a, w, cfg, 0);
  return out;
}

void gemm_configure_workspace_op(int64_t device, int64_t ws_bytes, int64_t n_counters) {
  gemm_configure_workspace((int)device, (size_t)ws_bytes, (int)n_counters);
}

void gemm_set_plan_op(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t cfg, int64_t splits) {
  gemm_set_plan((int)M, (int)N, (int)K, (int)epi, (int)cfg, (int)splits);
}
void gemm_clear_plans_op() { gemm_clear_plans(); }
void attn_fa_set_timeline_op(const std::optional<at::Tensor>& buf) {
  fa_tc_set_timeline(buf.has_value()
                         ? reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>())
                         : nullptr);
}

void gemm_set_timeline_op(const std::optional<at::Tensor>& buf) {
  if (buf.has_value()) {
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong, "timeline: int64 CUDA tensor");
    c10::cuda::CUDAGuard g(buf->device());
    gemm_set_timeline(reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>()));
  } else {
    gemm_set_timeline(nullptr);
  }
}
std::vector<int64_t> gemm_export_plans_op() {
  auto v = gemm_export_plans();
  return std::vector<int64_t>(v.begin(), v.end());
}

std::vector<int64_t> gemm_bf16_plan_op(int64_t M, int64_t N, int64_t K, int64_t epi,
                                       int64_t num_sm) {
  GemmPlan p = gemm_bf16_plan((int)M, (int)N, (int)K, (int)epi, (int)num_sm);
  return {p.cfg, p.splits};
}

// w_interleaved rows are [gate 64 | up 64] blocks (prepare with
// interleave_gate_up); output has w.size(0) / 2 columns.
void gemm_bf16_silu_mul_out(at::Tensor& out, const at::Tensor& a, const at::Tensor& w,
                            int64_t cfg) {
  CHECK_CUDA(a); CHECK_CUDA(w); CHECK_CUDA(out);
  CHECK_BF16(a); CHECK_BF16(w); CHECK_BF16(out);
  CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(w); CHECK_ROWMAJOR(out);
  TORCH_CHECK(a.size(1) == w.size(1), "gemm_bf16_silu_mul: K mismatch");
  TORCH_CHECK(w.size(0) % 128 == 0, "gemm_bf16_silu_mul: N must be a multiple of 128");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == w.size(0) / 2,
              "gemm_bf16_silu_mul: out shape");
  c10::cuda::CUDAGuard g(a.device());
  launch_gemm(out, a, w, kEpiSiluMul, cfg, 0);
}

int64_t gemm_bf16_config(int64_t M, int64_t N, int64_t K, int64_t epi) {
  return gemm_bf16_pick_config((int)M, (int)N, (int)K, (int)epi, 148);
}

WQParams make_wq(int64_t fmt, const at::Tensor& scales, double out_scale) {
  WQParams q{};
  q.scale_ld = (int)scales.size(1);
  q.out_scale = (float)out_scale;
  TORCH_CHECK(scales.is_cuda() && scales.is_contiguous() && scales.dim() == 2, "wq: scales 2-D");
  if (fmt == kWFp8) {
    TORCH_CHECK(scales.scalar_type() == at::kFloat, "fp8: fp32 block scales");
    q.scales_f32 = scales.data_ptr<float>();
  } else if (fmt == kWAwq) {
    TORCH_CHECK(scales.scalar_type() == at::kBFloat16 && scales.size(1) % 2 == 0,
                "awq: bf16 (scale, -zero*scale) pairs");
    q.scale_zero = reinterpret_cast<const __nv_bfloat162*>(scales.data_ptr());
    q.scale_ld = (int)scales.size(1) / 2;
  } else if (fmt == kWNvfp4) {
    TORCH_CHECK(scales.element_size() == 1, "nvfp4: e4m3 scales as 1-byte elements");
    q.scales_u8 = reinterpret_cast<const uint8_t*>(scales.data_ptr());
  } else {
    TORCH_CHECK(false, "unknown weight format ", fmt);
  }
  return q;
}

// Weight-only quantised GEMM for M <= 256 (fused dequant in the producer).
void gemm_wq_out(at::Tensor& out, const at::Tensor& a, const at::Tensor& w_raw, int64_t fmt,
                 const at::Tensor& scales, double out_scale, int64_t bn, int64_t splits) {
  CHECK_CUDA(a); CHECK_BF16(a); CHECK_BF16(out); CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(out);
  TORCH_CHECK(w_raw.is_cuda() && w_raw.dim() == 2 && w_raw.stride(1) == 1 &&
                  w_raw.element_size() == 1, "gemm_wq: raw weight must be 2-D bytes");
  const int M = (int)a.size(0), K = (int)a.size(1), N = (int)w_raw.size(0);
  const int rb = raw_row_bytes((int)fmt);
  TORCH_CHECK((int64_t)K * rb / 64 == w_raw.size(1), "gemm_wq: raw width does not match K");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm_wq: out shape");
  TORCH_CHECK(w_raw.stride(0) % 16 == 0, "gemm_wq: raw row stride must be 16B aligned");
  c10::cuda::CUDAGuard g(a.device());
  const WQParams q = make_wq(fmt, scales, out_scale);
  gemm_wq_launch(a.data_ptr(), w_raw.data_ptr(), out.data_ptr(), M, N, K, (int)a.stride(0),
                 (int)w_raw.stride(0), (int)out.stride(0), (int)fmt, q, (int)bn, (int)splits,
                 device_status_ptr(a.get_device()), cur_stream());
}

void dequant_weight(at::Tensor& out, const at::Tensor& w_raw, int64_t fmt, const at::Tensor& scales) {
  CHECK_BF16(out);
  TORCH_CHECK(out.is_contiguous() && w_raw.dim() == 2 && w_raw.element_size() == 1,
              "dequant_weight: shapes");
  const int N = (int)out.size(0), K = (int)out.size(1);
  c10::cuda::CUDAGuard g(out.device());
  const WQParams q = make_wq(fmt, scales, 1.0);
  dequant_weight_launch(w_raw.data_ptr(), w_raw.stride(0), out.data_ptr(), N, K, (int)fmt, q,
                        cur_stream());
}

void moe_topk(at::Tensor& w, at::Tensor& ids, const at::Tensor& logits, int64_t k,
              bool use_sigmoid, bool renorm, const c10::optional<at::Tensor>& bias) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "moe_topk: 2-D logits");
  const bool bf = logits.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf || logits.scalar_type() == at::kFloat, "moe_topk: bf16/fp32 logits");
  TORCH_CHECK(w.scalar_type() == at::kFloat && ids.scalar_type() == at::kInt, "moe_topk: outputs");
  TORCH_CHECK(w.numel() == logits.size(0) * k && ids.numel() == logits.size(0) * k, "moe_topk: sizes");
  c10::cuda::CUDAGuard g(logits.device());
  moe_topk_launch(logits.data_ptr(), bf, (int)logits.stride(0), (int)logits.size(0),
                  (int)logits.size(1), (int)k, use_sigmoid, renorm,
                  bias ? bias->data_ptr<float>() : nullptr, w.data_ptr<float>(), ids.data_ptr<int>(),
                  cur_stream());
}

// Fused router: fp32 logits of x [T, H] against wr [E, H] and the top-k in
// one kernel. logits [>= T, E] fp32 scratch; tile_ctr [>= ceil(T/8)] int32,
// zero before the first call (the kernel leaves it zero).
void moe_router(at::Tensor& w, at::Tensor& ids, const at::Tensor& x, const at::Tensor& wr,
                int64_t k, bool use_sigmoid, bool renorm, const c10::optional<at::Tensor>& bias,
                at::Tensor& logits, at::Tensor& tile_ctr) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(wr);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && wr.dim() == 2 && wr.is_contiguous() &&
              wr.size(1) == x.size(1), "moe_router: x [T, H], wr [E, H]");
  TORCH_CHECK(x.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(wr.data_ptr()) & 15) == 0, "moe_router: 16B-aligned rows");
  const int64_t T = x.size(0), E = wr.size(0);
  TORCH_CHECK(w.scalar_type() == at::kFloat && ids.scalar_type() == at::kInt &&
              w.numel() >= T * k && ids.numel() >= T * k, "moe_router: outputs");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.numel() >= T * E, "moe_router: logits scratch");
  TORCH_CHECK(tile_ctr.scalar_type() == at::kInt && tile_ctr.numel() >= (T + 7) / 8,
              "moe_router: tile counters");
  c10::cuda::CUDAGuard g(x.device());
  moe_router_launch(x.data_ptr(), (int)x.stride(0), wr.data_ptr(), (int)T, (int)E, (int)x.size(1),
                    (int)k, use_sigmoid, renorm, bias ? bias->data_ptr<float>() : nullptr,
                    logits.data_ptr<float>(), tile_ctr.data_ptr<int>(), w.data_ptr<float>(),
                    ids.data_ptr<int>(), cur_stream());
}

// Expert-sort the (token, slot) pairs of experts [e_base, e_base + E).
void moe_permute(const at::Tensor& ids, int64_t E, int64_t e_base, const c10::optional<at::Tensor>& x,
                 const c10::optional<at::Tensor>& x_perm, at::Tensor& counts, at::Tensor& offsets,
                 at::Tensor& rank_scratch, at::Tensor& pos, at::Tensor& src_row, int64_t align) {
  CHECK_CUDA(ids);
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.dim() == 2 && ids.is_contiguous(), "ids [T, k] int32");
  const int T = (int)ids.size(0), k = (int)ids.size(1);
  TORCH_CHECK(counts.numel() >= E && offsets.numel() >= E + 1, "moe_permute: counts/offsets");
  TORCH_CHECK(align >= 1, "moe_permute: align >= 1");
  const int64_t padded = (int64_t)T * k + E * (align - 1);
  TORCH_CHECK(rank_scratch.numel() >= T * k && pos.numel() >= T * k && src_row.numel() >= padded,
              "moe_permute: scratch sizes");
  int H = 0;
  if (x) {
    CHECK_BF16((*x));
    TORCH_CHECK(x_perm && x->is_contiguous() && x_perm->is_contiguous(), "moe_permute: x / x_perm");
    H = (int)x->size(1);
    TORCH_CHECK(H % 8 == 0 && x_perm->size(1) == H && x_perm->size(0) >= padded, "moe_permute: H");
  }
  c10::cuda::CUDAGuard g(ids.device());
  moe_permute_launch(ids.data_ptr<int>(), T, k, (int)E, (int)e_base, x ? x->data_ptr() : nullptr, H,
                     x_perm ? x_perm->data_ptr() : nullptr, counts.data_ptr<int>(),
                     offsets.data_ptr<int>(), rank_scratch.data_ptr<int>(), pos.data_ptr<int>(),
                     src_row.data_ptr<int>(), cur_stream(), (int)align);
}

void moe_combine(at::Tensor& out, const at::Tensor& y, const at::Tensor& pos, const at::Tensor& w,
                 const c10::optional<at::Tensor>& shared, double shared_scale) {
  CHECK_CUDA(y); CHECK_BF16(y); CHECK_BF16(out);
  TORCH_CHECK(pos.scalar_type() == at::kInt && w.scalar_type() == at::kFloat, "moe_combine: types");
  const int T = (int)pos.size(0), k = (int)pos.size(1), H = (int)out.size(1);
  TORCH_CHECK(out.is_contiguous() && y.is_contiguous() && y.size(1) == H && H % 2 == 0, "moe_combine");
  c10::cuda::CUDAGuard g(y.device());
  moe_combine_launch(y.data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(), T, k, H,
                     shared ? shared->data_ptr() : nullptr, (float)shared_scale, out.data_ptr(),
                     cur_stream());
}

// Grouped expert GEMM over expert-sorted rows.
void gemm_grouped_out(at::Tensor& out, const at::Tensor& x, const at::Tensor& w_stk, int64_t E,
                      int64_t N, const at::Tensor& row_off, at::Tensor& tile_off, int64_t fmt,
                      const c10::optional<at::Tensor>& scales, double out_scale, int64_t bn) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(out); CHECK_ROWMAJOR(x); CHECK_ROWMAJOR(out);
  TORCH_CHECK(row_off.scalar_type() == at::kInt && tile_off.scalar_type() == at::kInt &&
                  row_off.numel() >= E + 1 && tile_off.numel() >= E + 1, "gemm_grouped: offsets");
  TORCH_CHECK(w_stk.dim() == 2 && w_stk.stride(1) == 1 && w_stk.size(0) == E * N, "gemm_grouped: W");
  const int K = (int)x.size(1);
  WQParams q{};
  if (fmt != kWBf16) {
    TORCH_CHECK(scales, "gemm_grouped: quantised weights need scales");
    q = make_wq(fmt, *scales, out_scale);
    TORCH_CHECK((int64_t)K * raw_row_bytes((int)fmt) / 64 == w_stk.size(1), "gemm_grouped: raw width");
  } else {
    CHECK_BF16(w_stk);
    TORCH_CHECK(w_stk.size(1) == K, "gemm_grouped: K");
  }
  TORCH_CHECK(out.size(0) >= x.size(0) && out.size(1) == N, "gemm_grouped: out shape");
  c10::cuda::CUDAGuard g(x.device());
  gemm_grouped_launch(x.data_ptr(), w_stk.data_ptr(), out.data_ptr(), (int)x.size(0), (int)E,
                      (int)N, K, (int)x.stride(0), (int)w_stk.stride(0), (int)out.stride(0),
                      row_off.data_ptr<int>(), tile_off.data_ptr<int>(), (int)fmt, q, (int)bn,
                      device_status_ptr(x.get_device()), cur_stream());
}

// Block-scaled FP8 (W8A8): activation quantisation and the kind::f8f6f4 GEMMs.
void quant_fp8_act(const at::Tensor& x, at::Tensor& xq, at::Tensor& sa) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_ROWMAJOR(x);
  TORCH_CHECK(xq.is_cuda() && xq.element_size() == 1 && xq.dim() == 2 && xq.stride(1) == 1 &&
                  xq.size(0) == x.size(0) && xq.size(1) == x.size(1), "quant_fp8_act: xq");
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sa.dim() == 2 && sa.stride(1) == 1 &&
                  sa.size(0) == (x.size(1) + 127) / 128 && sa.size(1) >= x.size(0),
              "quant_fp8_act: sa must be fp32 [ceil(K/128), >= M]");
  c10::cuda::CUDAGuard g(x.device());
  quant_fp8_act_launch(x.data_ptr(), (int)x.stride(0), (int)x.size(0), (int)x.size(1),
                       xq.data_ptr(), (int)xq.stride(0), sa.data_ptr<float>(), (int)sa.stride(0),
                       cur_stream());
}

void gemm_fp8_out(at::Tensor& out, const at::Tensor& xq, const at::Tensor& sa,
                  const at::Tensor& wq, const at::Tensor& sw, int64_t bn) {
  CHECK_BF16(out); CHECK_ROWMAJOR(out);
  TORCH_CHECK(xq.is_cuda() && xq.element_size() == 1 && xq.dim() == 2 && xq.stride(1) == 1,
              "gemm_fp8: xq must be 2-D e4m3 bytes");
  TORCH_CHECK(wq.is_cuda() && wq.element_size() == 1 && wq.dim() == 2 && wq.stride(1) == 1 &&
                  wq.size(1) == xq.size(1), "gemm_fp8: wq must be 2-D e4m3 bytes [N, K]");
  const int M = (int)xq.size(0), K = (int)xq.size(1), N = (int)wq.size(0);
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sa.dim() == 2 && sa.stride(1) == 1 &&
                  sa.size(0) == (K + 127) / 128 && sa.size(1) >= M, "gemm_fp8: sa shape");
  TORCH_CHECK(sw.scalar_type() == at::kFloat && sw.dim() == 2 && sw.stride(1) == 1 &&
                  sw.size(0) == (N + 127) / 128 && sw.size(1) >= (K + 127) / 128,
              "gemm_fp8: sw must be fp32 [ceil(N/128), ceil(K/128)]");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm_fp8: out shape");
  c10::cuda::CUDAGuard g(xq.device());
  gemm_fp8_launch(xq.data_ptr(), sa.data_ptr<float>(), (int)sa.stride(0), wq.data_ptr(),
                  sw.data_ptr<float>(), (int)sw.stride(0), out.data_ptr(), M, N, K,
                  (int)xq.stride(0), (int)wq.stride(0), (int)out.stride(0), (int)bn,
                  device_status_ptr(xq.get_device()), cur_stream());
}

void gemm_fp8_grouped_out(at::Tensor& out, const at::Tensor& xq, const at::Tensor& sa,
                          const at::Tensor& w_stk, const at::Tensor& sw, int64_t E, int64_t N,
                          const at::Tensor& row_off, at::Tensor& tile_off, int64_t bn) {
  CHECK_BF16(out); CHECK_ROWMAJOR(out);
  TORCH_CHECK(xq.is_cuda() && xq.element_size() == 1 && xq.dim() == 2 && xq.stride(1) == 1,
              "gemm_fp8_grouped: xq");
  TORCH_CHECK(w_stk.element_size() == 1 && w_stk.dim() == 2 && w_stk.stride(1) == 1 &&
                  w_stk.size(0) == E * N && w_stk.size(1) == xq.size(1), "gemm_fp8_grouped: W");
  TORCH_CHECK(row_off.scalar_type() == at::kInt && tile_off.scalar_type() == at::kInt &&
                  row_off.numel() >= E + 1 && tile_off.numel() >= E + 1,
              "gemm_fp8_grouped: offsets");
  const int rows = (int)xq.size(0), K = (int)xq.size(1);
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sa.dim() == 2 && sa.stride(1) == 1 &&
                  sa.size(0) == (K + 127) / 128 && sa.size(1) >= rows, "gemm_fp8_grouped: sa");
  TORCH_CHECK(sw.scalar_type() == at::kFloat && sw.dim() == 2 && sw.stride(1) == 1 &&
                  sw.size(0) == E * N / 128 && sw.size(1) >= (K + 127) / 128,
              "gemm_fp8_grouped: sw must be fp32 [E * N / 128, ceil(K/128)]");
  TORCH_CHECK(out.size(0) >= rows && out.size(1) == N, "gemm_fp8_grouped: out shape");
  c10::cuda::CUDAGuard g(xq.device());
  gemm_fp8_grouped_launch(xq.data_ptr(), sa.data_ptr<float>(), (int)sa.stride(0), w_stk.data_ptr(),
                          sw.data_ptr<float>(), (int)sw.stride(0), out.data_ptr(), rows, (int)E,
                          (int)N, K, (int)xq.stride(0), (int)w_stk.stride(0), (int)out.stride(0),
                          row_off.data_ptr<int>(), tile_off.data_ptr<int>(), (int)bn,
                          device_status_ptr(xq.get_device()), cur_stream());
}

// NVFP4 W4A4 (kind::mxf4nvf4): activation quantisation and the GEMMs. Scale
// tensors are bytes in the 128-row x 4-scale atom order [rows/128][K/64][512].
void quant_nvfp4_act(const at::Tensor& x, at::Tensor& xq, at::Tensor& sf, at::Tensor& rs,
                     const c10::optional<at::Tensor>& n_rows) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_ROWMAJOR(x);
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 64 == 0, "quant_nvfp4_act: K % 64");
  TORCH_CHECK(xq.element_size() == 1 && xq.dim() == 2 && xq.size(0) >= M && xq.size(1) == K / 2 &&
                  xq.stride(1) == 1, "quant_nvfp4_act: xq [M, K/2] bytes");
  TORCH_CHECK(sf.element_size() == 1 && sf.is_contiguous() &&
                  sf.numel() >= (M + 127) / 128 * (K / 64) * 512, "quant_nvfp4_act: sf atoms");
  TORCH_CHECK(rs.scalar_type() == at::kFloat && rs.numel() >= M, "quant_nvfp4_act: rs");
  c10::cuda::CUDAGuard g(x.device());
  quant_nvfp4_act_launch(x.data_ptr(), (int)x.stride(0), (int)M, (int)K, xq.data_ptr(),
                         (int)xq.stride(0), sf.data_ptr(), rs.data_ptr<float>(), cur_stream(),
                         n_rows ? n_rows->data_ptr<int>() : nullptr);
}

void gemm_nvfp4_out(at::Tensor& out, const at::Tensor& xq, const at::Tensor& sfa,
                    const at::Tensor& rs, const at::Tensor& wq, const at::Tensor& sfw, double g,
                    int64_t swap) {
  CHECK_BF16(out); CHECK_ROWMAJOR(out);
  TORCH_CHECK(xq.element_size() == 1 && wq.element_size() == 1 && xq.dim() == 2 && wq.dim() == 2 &&
                  xq.stride(1) == 1 && wq.stride(1) == 1 && xq.size(1) == wq.size(1),
              "gemm_nvfp4: packed operands [rows, K/2]");
  const int M = (int)xq.size(0), N = (int)wq.size(0), K = (int)xq.size(1) * 2;
  TORCH_CHECK(sfa.numel() >= (int64_t)(M + 127) / 128 * (K / 64) * 512 &&
                  sfw.numel() >= (int64_t)(N + 127) / 128 * (K / 64) * 512, "gemm_nvfp4: scale atoms");
  TORCH_CHECK(rs.scalar_type() == at::kFloat && rs.numel() >= M, "gemm_nvfp4: rs");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm_nvfp4: out shape");
  c10::cuda::CUDAGuard gd(xq.device());
  gemm_nvfp4_launch(xq.data_ptr(), sfa.data_ptr(), rs.data_ptr<float>(), wq.data_ptr(),
                    sfw.data_ptr(), (float)g, out.data_ptr(), M, N, K, (int)xq.stride(0),
                    (int)wq.stride(0), (int)out.stride(0), (int)swap,
                    device_status_ptr(xq.get_device()), cur_stream());
}

void gemm_nvfp4_grouped_out(at::Tensor& out, const at::Tensor& xq, const at::Tensor& sfx,
                            const at::Tensor& rs, const at::Tensor& w_stk, const at::Tensor& sfw,
                            double g, int64_t E, int64_t N, const at::Tensor& row_off,
                            at::Tensor& tile_off) {
  CHECK_BF16(out); CHECK_ROWMAJOR(out);
  TORCH_CHECK(xq.element_size() == 1 && w_stk.element_size() == 1 && xq.size(1) == w_stk.size(1) &&
                  w_stk.size(0) == E * N, "gemm_nvfp4_grouped: operands");
  TORCH_CHECK(row_off.scalar_type() == at::kInt && tile_off.scalar_type() == at::kInt &&
                  row_off.numel() >= E + 1 && tile_off.numel() >= E + 1, "gemm_nvfp4_grouped: offsets");
  const int rows = (int)xq.size(0), K = (int)xq.size(1) * 2;
  TORCH_CHECK(out.size(0) >= rows && out.size(1) == N, "gemm_nvfp4_grouped: out shape");
  c10::cuda::CUDAGuard gd(xq.device());
  gemm_nvfp4_grouped_launch(xq.data_ptr(), sfx.data_ptr(), rs.data_ptr<float>(), w_stk.data_ptr(),
                            sfw.data_ptr(), (float)g, out.data_ptr(), rows, (int)E, (int)N, K,
                            (int)xq.stride(0), (int)w_stk.stride(0), (int)out.stride(0),
                            row_off.data_ptr<int>(), tile_off.data_ptr<int>(),
                            device_status_ptr(xq.get_device()), cur_stream());
}

void gumbel_argmax(at::Tensor& ids, at::Tensor& vals, const at::Tensor& logits,
                   const at::Tensor& temperature, const at::Tensor& seeds, int64_t offset,
                   int64_t id_offset, const c10::optional<at::Tensor>& row_offsets) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "gumbel_argmax: 2-D logits");
  const bool bf = logits.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf || logits.scalar_type() == at::kFloat, "gumbel_argmax: bf16/fp32 logits");
  TORCH_CHECK(temperature.scalar_type() == at::kFloat && seeds.scalar_type() == at::kLong,
              "gumbel_argmax: fp32 temperature, int64 seeds");
  c10::cuda::CUDAGuard g(logits.device());
  gumbel_argmax_launch(logits.data_ptr(), bf, (int)logits.size(0), (int)logits.size(1),
                       (int)logits.stride(0), temperature.data_ptr<float>(),
                       seeds.data_ptr<int64_t>(), (uint64_t)offset,
                       row_offsets ? row_offsets->data_ptr<int64_t>() : nullptr, (int)id_offset,
                       ids.data_ptr<int>(), vals.data_ptr<float>(), cur_stream());
}

void topk_candidates(at::Tensor& vals, at::Tensor& ids, const at::Tensor& logits, int64_t K,
                     int64_t id_offset) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "topk_candidates: 2-D logits");
  const bool bf = logits.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf || logits.scalar_type() == at::kFloat, "topk_candidates: bf16/fp32 logits");
  TORCH_CHECK(vals.numel() >= logits.size(0) * K && ids.numel() >= logits.size(0) * K,
              "topk_candidates: outputs");
  c10::cuda::CUDAGuard g(logits.device());
  topk_candidates_launch(logits.data_ptr(), bf, (int)logits.size(0), (int)logits.size(1),
                         (int)logits.stride(0), (int)K, (int)id_offset, vals.data_ptr<float>(),
                         ids.data_ptr<int>(), cur_stream());
}

void sample_candidates(at::Tensor& out, const at::Tensor& cand_v, const at::Tensor& cand_i,
                       const at::Tensor& temperature, const at::Tensor& top_k,
                       const at::Tensor& top_p, const at::Tensor& seeds, int64_t offset) {
  CHECK_CUDA(cand_v);
  TORCH_CHECK(cand_v.dim() == 2 && cand_v.is_contiguous() && cand_i.is_contiguous(),
              "sample_candidates: [rows, C]");
  c10::cuda::CUDAGuard g(cand_v.device());
  sample_candidates_launch(cand_v.data_ptr<float>(), cand_i.data_ptr<int>(), (int)cand_v.size(0),
                           (int)cand_v.size(1), temperature.data_ptr<float>(),
                           top_k.data_ptr<int>(), top_p.data_ptr<float>(),
                           seeds.data_ptr<int64_t>(), (uint64_t)offset, out.data_ptr<int>(),
                           cur_stream());
}

void causal_conv1d(at::Tensor& y, const at::Tensor& x, const at::Tensor& w,
                   const c10::optional<at::Tensor>& bias, at::Tensor& state, const at::Tensor& cu,
                   const at::Tensor& slots, bool silu, bool write_state) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(y); CHECK_BF16(w);
  TORCH_CHECK(x.stride(1) == 1 && y.stride(1) == 1 && w.is_contiguous() && w.dim() == 2,
              "causal_conv1d: layouts");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.dim() == 3 &&
                  state.size(1) == x.size(1) && state.size(2) == w.size(1) - 1,
              "causal_conv1d: state [slots, C, W-1] fp32");
  TORCH_CHECK(cu.scalar_type() == at::kInt && slots.scalar_type() == at::kInt, "int32 metadata");
  c10::cuda::CUDAGuard g(x.device());
  causal_conv1d_launch(x.data_ptr(), (int)x.stride(0), w.data_ptr(),
                       bias ? bias->data_ptr() : nullptr, y.data_ptr(), (int)y.stride(0),
                       state.data_ptr<float>(), cu.data_ptr<int>(), slots.data_ptr<int>(),
                       (int)slots.numel(), (int)x.size(1), (int)w.size(1), silu, write_state,
                       cur_stream());
}

void gdn_recurrent(at::Tensor& o, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                   const at::Tensor& a, const at::Tensor& b, const at::Tensor& A_log,
                   const at::Tensor& dt_bias, at::Tensor& state, const at::Tensor& cu,
                   const at::Tensor& slots, int64_t HK, int64_t HV, bool reset_state,
                   bool write_state, bool chunked, const c10::optional<at::Tensor>& has_init) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_BF16(k); CHECK_BF16(v); CHECK_BF16(a); CHECK_BF16(b);
  CHECK_BF16(o);
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat,
              "gdn: fp32 A_log / dt_bias");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.dim() == 4,
              "gdn: state [slots, HV, DV, DK] fp32");
  const int DK = (int)(q.size(1) / HK), DV = (int)(v.size(1) / HV);
  TORCH_CHECK(state.size(1) == HV && state.size(2) == DV && state.size(3) == DK, "gdn: state dims");
  // Slots may be padded apart (paged state); each slot's [HV, DV, DK] block is dense and
  // every slot starts on 16 bytes (the kernels read the state as float4 / float2).
  TORCH_CHECK(state.stride(3) == 1 && state.stride(2) == DK && state.stride(1) == (int64_t)DV * DK &&
                  state.stride(0) >= (int64_t)HV * DV * DK && state.stride(0) % 4 == 0 &&
                  reinterpret_cast<uintptr_t>(state.data_ptr()) % 16 == 0,
              "gdn: each state slot must be a dense 16-byte aligned [HV, DV, DK] block");
  TORCH_CHECK(cu.scalar_type() == at::kInt && slots.scalar_type() == at::kInt &&
                  cu.is_contiguous() && slots.is_contiguous() && cu.numel() >= slots.numel() + 1,
              "gdn: cu [nseq + 1] / slots [nseq] int32");
  const unsigned char* init_ptr = nullptr;
  if (has_init.has_value()) {
    const at::Tensor& hi = *has_init;
    TORCH_CHECK(hi.is_cuda() && (hi.scalar_type() == at::kBool || hi.scalar_type() == at::kByte) &&
                    hi.is_contiguous() && hi.numel() == slots.numel(),
                "gdn: has_init [nseq] bool");
    init_ptr = reinterpret_cast<const unsigned char*>(hi.data_ptr());
  }
  TORCH_CHECK(a.stride(0) == b.stride(0) && a.stride(1) == 1 && b.stride(1) == 1, "gdn: a/b layout");
  TORCH_CHECK(q.stride(1) == 1 && k.stride(1) == 1 && v.stride(1) == 1 && o.stride(1) == 1,
              "gdn: q / k / v / o rows must have unit inner stride");
  GdnParams p{};
  p.q = (const __nv_bfloat16*)q.data_ptr(); p.k = (const __nv_bfloat16*)k.data_ptr();
  p.v = (const __nv_bfloat16*)v.data_ptr(); p.a = (const __nv_bfloat16*)a.data_ptr();
  p.b = (const __nv_bfloat16*)b.data_ptr(); p.A_log = A_log.data_ptr<float>();
  p.dt_bias = dt_bias.data_ptr<float>(); p.o = (__nv_bfloat16*)o.data_ptr();
  p.state = state.data_ptr<float>(); p.cu = cu.data_ptr<int>(); p.slots = slots.data_ptr<int>();
  p.ldq = (int)q.stride(0); p.ldk = (int)k.stride(0); p.ldv = (int)v.stride(0);
  p.ldab = (int)a.stride(0); p.ldo = (int)o.stride(0);
  p.HK = (int)HK; p.HV = (int)HV; p.reset_state = reset_state ? 1 : 0;
  p.write_state = write_state ? 1 : 0;
  p.ld_state = state.stride(0);
  p.has_init = init_ptr;
  c10::cuda::CUDAGuard g(q.device());
  if (chunked) {
    TORCH_CHECK(gdn_chunk_supported(DK, DV), "gdn: the chunked form needs DK = DV = 128");
    gdn_chunk_launch(p, (int)slots.numel(), DK, DV, cur_stream());
  } else {
    gdn_recurrent_launch(p, (int)slots.numel(), DK, DV, cur_stream());
  }
}

void gated_rmsnorm(at::Tensor& o, const at::Tensor& z, const at::Tensor& w, int64_t H, double eps) {
  CHECK_CUDA(o); CHECK_BF16(o); CHECK_BF16(z); CHECK_BF16(w);
  const int D = (int)w.numel();
  TORCH_CHECK(o.size(1) == H * D && o.stride(1) == 1 && z.stride(1) == 1, "gated_rmsnorm: layout");
  c10::cuda::CUDAGuard g(o.device());
  gated_rmsnorm_launch(o.data_ptr(), (int)o.stride(0), z.data_ptr(), (int)z.stride(0),
                       w.data_ptr(), (int)o.size(0), (int)H, D, (float)eps, cur_stream());
}

void rejection_sample(at::Tensor& out_tokens, at::Tensor& num_out, const at::Tensor& target_logits,
                      const at::Tensor& draft_logits, const at::Tensor& draft_ids,
                      const at::Tensor& temperature, const at::Tensor& seeds, int64_t offset) {
  CHECK_CUDA(target_logits); CHECK_BF16(target_logits); CHECK_BF16(draft_logits);
  TORCH_CHECK(target_logits.dim() == 3 && draft_logits.dim() == 3 && target_logits.is_contiguous() &&
                  draft_logits.is_contiguous(), "rejection_sample: [rows, k(+1), V] contiguous");
  const int rows = (int)draft_ids.size(0), k = (int)draft_ids.size(1);
  const int V = (int)target_logits.size(2);
  TORCH_CHECK(target_logits.size(1) == k + 1 && draft_logits.size(1) == k &&
                  draft_logits.size(2) == V, "rejection_sample: shapes");
  TORCH_CHECK(draft_ids.scalar_type() == at::kInt && draft_ids.is_contiguous(), "draft ids int32");
  c10::cuda::CUDAGuard g(target_logits.device());
  rejection_sample_launch(target_logits.data_ptr(), draft_logits.data_ptr(),
                          draft_ids.data_ptr<int>(), rows, k, V, temperature.data_ptr<float>(),
                          seeds.data_ptr<int64_t>(), (uint64_t)offset, out_tokens.data_ptr<int>(),
                          num_out.data_ptr<int>(), cur_stream());
}

void rms_norm(at::Tensor& out, const at::Tensor& x, const at::Tensor& w, double eps) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w); CHECK_BF16(out);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1, "rms_norm: 2-D rows");
  c10::cuda::CUDAGuard g(x.device());
  rms_norm_launch(out.data_ptr(), (int)out.stride(0), x.data_ptr(), (int)x.stride(0), w.data_ptr(),
                  (int)x.size(0), (int)x.size(1), (float)eps, cur_stream());
}

void fused_add_rms_norm(at::Tensor& x, at::Tensor& residual, const at::Tensor& w, double eps) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(residual); CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && residual.stride(1) == 1,
              "fused_add_rms_norm: 2-D rows");
  TORCH_CHECK(x.sizes() == residual.sizes(), "fused_add_rms_norm: shape mismatch");
  c10::cuda::CUDAGuard g(x.device());
  fused_add_rms_norm_launch(x.data_ptr(), (int)x.stride(0), residual.data_ptr(),
                            (int)residual.stride(0), w.data_ptr(), (int)x.size(0), (int)x.size(1),
                            (float)eps, cur_stream());
}

void rope_kv_write(at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& cos_sin,
                   at::Tensor& k_cache, at::Tensor& v_cache, const at::Tensor& slot_mapping,
                   int64_t num_q_heads, int64_t num_kv_heads, const c10::optional<at::Tensor>& q_norm,
                   const c10::optional<at::Tensor>& k_norm, double eps) {
  CHECK_CUDA(qkv); CHECK_BF16(qkv); CHECK_BF16(k_cache); CHECK_BF16(v_cache);
  TORCH_CHECK(positions.scalar_type() == at::kLong && slot_mapping.scalar_type() == at::kLong,
              "rope_kv_write: positions / slot_mapping must be int64");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin fp32");
  TORCH_CHECK(qkv.is_contiguous(), "rope_kv_write: contiguous qkv required");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.dim() == 4, "k_cache must be [blocks, Hkv, BS, D]");
  for (const at::Tensor* c : {&k_cache, &v_cache})
    TORCH_CHECK(c->stride(3) == 1 && c->stride(2) == c->size(3) &&
                    c->stride(1) == c->size(2) * c->size(3),
                "rope_kv_write: cache blocks must be dense [Hkv, BS, D]");
  TORCH_CHECK(k_cache.stride(0) == v_cache.stride(0), "rope_kv_write: K/V block strides differ");
  const int T = (int)qkv.size(0);
  const int D = (int)k_cache.size(3);
  const int BS = (int)k_cache.size(2);
  TORCH_CHECK(qkv.size(1) == (num_q_heads + 2 * num_kv_heads) * D, "rope_kv_write: qkv width");
  TORCH_CHECK(positions.numel() >= T && slot_mapping.numel() >= T, "rope_kv_write: lengths");
  c10::cuda::CUDAGuard g(qkv.device());
  rope_kv_write_launch(qkv.data_ptr(), positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(),
                       k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr<int64_t>(),
                       q_norm ? q_norm->data_ptr() : nullptr, k_norm ? k_norm->data_ptr() : nullptr,
                       T, (int)num_q_heads, (int)num_kv_heads, D, BS, (float)eps,
                       (int)cos_sin.size(1), k_cache.stride(0), cur_stream());
}

void kv_cache_write(const at::Tensor& k, const at::Tensor& v, at::Tensor& k_cache,
                    at::Tensor& v_cache, const at::Tensor& slots) {
  CHECK_CUDA(k); CHECK_BF16(k); CHECK_BF16(v); CHECK_BF16(k_cache); CHECK_BF16(v_cache);
  TORCH_CHECK(k.dim() == 3 && v.dim() == 3 && k.stride(2) == 1 && v.stride(2) == 1 &&
                  k.stride(1) == k.size(2) && v.stride(1) == v.size(2),
              "kv_cache_write: k/v must be [T, Hkv, D] with dense heads");
  TORCH_CHECK(slots.scalar_type() == at::kLong, "kv_cache_write: int64 slot mapping");
  for (const at::Tensor* c : {&k_cache, &v_cache})
    TORCH_CHECK(c->dim() == 4 && c->stride(3) == 1 && c->stride(2) == c->size(3) &&
                    c->stride(1) == c->size(2) * c->size(3),
                "kv_cache_write: cache blocks must be dense [Hkv, BS, D]");
  TORCH_CHECK(k.size(2) % 8 == 0 && k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0,
              "kv_cache_write: 16-byte aligned rows");
  c10::cuda::CUDAGuard g(k.device());
  kv_cache_write_launch(k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), k_cache.data_ptr(),
                        v_cache.data_ptr(), slots.data_ptr<int64_t>(), (int)k.size(0),
                        (int)k.size(1), (int)k.size(2), (int)k_cache.size(2), k_cache.stride(0),
                        cur_stream());
}

void paged_attention(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                     const at::Tensor& v_cache, const at::Tensor& block_table,
                     const at::Tensor& seq_lens, const at::Tensor& cu_q, int64_t max_q_len,
                     double scale, int64_t window, const c10::optional<at::Tensor>& sinks,
                     bool decode, int64_t num_splits, const c10::optional<at::Tensor>& part_o,
                     const c10::optional<at::Tensor>& part_ml) {
  CHECK_CUDA(q); CHECK_BF16(q); CHECK_BF16(out); CHECK_BF16(k_cache); CHECK_BF16(v_cache);
  TORCH_CHECK(q.dim() == 3 && out.dim() == 3, "paged_attention: q/out must be [T, H, D]");
  TORCH_CHECK(q.stride(2) == 1 && q.stride(1) == q.size(2), "paged_attention: q head layout");
  TORCH_CHECK(out.stride(2) == 1 && out.stride(1) == out.size(2), "paged_attention: out layout");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.dim() == 4, "paged_attention: caches [blocks, Hkv, BS, D]");
  // Each (block, head) must be a dense BS x D tile; blocks may be strided
  // (e.g. K and V interleaved per block in one allocation).
  for (const at::Tensor* c : {&k_cache, &v_cache}) {
    TORCH_CHECK(c->stride(3) == 1 && c->stride(2) == c->size(3) &&
                    c->stride(1) == c->size(2) * c->size(3),
                "paged_attention: cache blocks must be dense [Hkv, BS, D]");
    TORCH_CHECK(c->stride(0) % 8 == 0, "paged_attention: cache block stride must be 16B aligned");
  }
  TORCH_CHECK(k_cache.stride(0) == v_cache.stride(0), "paged_attention: K/V block strides differ");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  cu_q.scalar_type() == at::kInt,
              "paged_attention: int32 metadata");
  TORCH_CHECK(block_table.is_contiguous() && seq_lens.is_contiguous() && cu_q.is_contiguous(),
              "paged_attention: contiguous metadata");
  TORCH_CHECK(q.stride(0) % 8 == 0, "paged_attention: q token stride must be 16B aligned");
  AttnArgs a{};
  a.q = q.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.out = out.data_ptr();
  a.block_table = block_table.data_ptr<int>();
  a.seq_lens = seq_lens.data_ptr<int>();
  a.cu_q = cu_q.data_ptr<int>();
  a.sinks = sinks ? sinks->data_ptr<float>() : nullptr;
  a.part_o = part_o ? part_o->data_ptr<float>() : nullptr;
  a.part_ml = part_ml ? part_ml->data_ptr<float>() : nullptr;
  a.num_seqs = (int)seq_lens.size(0);
  a.num_tokens = (int)q.size(0);
  a.Hq = (int)q.size(1);
  a.Hkv = (int)k_cache.size(1);
  a.head_dim = (int)q.size(2);
  a.block_size = (int)k_cache.size(2);
  a.max_blocks = (int)block_table.size(1);
  a.num_blocks = (int)k_cache.size(0);
  a.max_q_len = (int)max_q_len;
  a.window = (int)window;
  a.q_stride_t = (int)q.stride(0);
  a.o_stride_t = (int)out.stride(0);
  a.scale = (float)scale;
  a.decode = decode;
  a.num_splits = (int)num_splits;
  a.kv_block_stride = k_cache.stride(0);
  if (a.num_splits > 1) {
    TORCH_CHECK(part_o && part_ml, "split-KV decode needs part_o / part_ml");
    TORCH_CHECK(part_o->numel() >= (int64_t)a.num_splits * a.num_tokens * a.Hq * a.head_dim,
                "part_o too small");
    TORCH_CHECK(part_ml->numel() >= (int64_t)a.num_splits * a.num_tokens * a.Hq * 2,
                "part_ml too small");
  }
  c10::cuda::CUDAGuard g(q.device());
  paged_attention_launch(a, cur_stream());
}

// Fused TP all-reduce + residual add + RMSNorm over peer-mapped symmetric
// buffers (addresses from the symmetric-memory rendezvous, one per rank).
// Multicast addresses [stage, res, out] (NVLS) or an empty list.
static void set_mc(ArRmsNormParams& p, const std::vector<int64_t>& mc_ptrs) {
  TORCH_CHECK(mc_ptrs.empty() || mc_ptrs.size() == 3, "ar_rmsnorm: mc_ptrs = [stage, res, out]");
  if (mc_ptrs.size() == 3) {
    TORCH_CHECK((mc_ptrs[0] | mc_ptrs[1] | mc_ptrs[2]) % 16 == 0 && mc_ptrs[0] && mc_ptrs[1] &&
                mc_ptrs[2], "ar_rmsnorm: multicast addresses");
    p.mc_stage = reinterpret_cast<const __nv_bfloat16*>(mc_ptrs[0]);
    p.mc_res = reinterpret_cast<__nv_bfloat16*>(mc_ptrs[1]);
    p.mc_out = reinterpret_cast<__nv_bfloat16*>(mc_ptrs[2]);
  }
}

void ar_rmsnorm(const std::vector<int64_t>& stage_ptrs, const std::vector<int64_t>& res_ptrs,
                const std::vector<int64_t>& out_ptrs, const std::vector<int64_t>& flag_ptrs,
                int64_t rank, int64_t T, int64_t H, const at::Tensor& w, double eps,
                int64_t timeout_ms, int64_t grid, const std::vector<int64_t>& mc_ptrs) {
  const int W = (int)stage_ptrs.size();
  TORCH_CHECK(W == 2 || W == 4 || W == 8, "ar_rmsnorm: world size must be 2, 4 or 8");
  TORCH_CHECK((int)res_ptrs.size() == W && (int)out_ptrs.size() == W && (int)flag_ptrs.size() == W,
              "ar_rmsnorm: pointer lists must have one entry per rank");
  TORCH_CHECK(rank >= 0 && rank < W, "ar_rmsnorm: bad rank");
  CHECK_CUDA(w); CHECK_BF16(w);
  TORCH_CHECK(w.numel() == H && H % 8 == 0, "ar_rmsnorm: weight size / H % 8");
  ArRmsNormParams p{};
  for (int q = 0; q < W; ++q) {
    p.stage_peer[q] = reinterpret_cast<const __nv_bfloat16*>(stage_ptrs[q]);
    p.res_peer[q] = reinterpret_cast<__nv_bfloat16*>(res_ptrs[q]);
    p.out_peer[q] = reinterpret_cast<__nv_bfloat16*>(out_ptrs[q]);
    p.flags_peer[q] = reinterpret_cast<uint32_t*>(flag_ptrs[q]);
    TORCH_CHECK((stage_ptrs[q] | res_ptrs[q] | out_ptrs[q]) % 16 == 0, "ar_rmsnorm: 16B alignment");
  }
  p.flags_local = p.flags_peer[rank];
  p.res_local = p.res_peer[rank];
  p.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.rank = (int)rank;
  p.world = W;
  p.T = (int)T;
  p.H = (int)H;
  p.eps = (float)eps;
  p.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
  p.err = device_status_ptr(w.get_device());
  set_mc(p, mc_ptrs);
  c10::cuda::CUDAGuard g(w.device());
  ar_rmsnorm_launch(p, (int)grid, cur_stream());
}

// Expert-parallel exchange over peer memory. `bufs` lists, per rank, the
// addresses of (recv_x, recv_meta, back_y, pad) from the symmetric-memory
// rendezvous: bufs[4 * r + i].
static EpParams make_ep(const std::vector<int64_t>& bufs, int64_t rank, int64_t H, int64_t k,
                        int64_t E_local, int64_t T_cap, int64_t timeout_ms, int device) {
  const int W = (int)bufs.size() / 4;
  TORCH_CHECK((int)bufs.size() == 4 * W && W >= 2 && W <= kMaxRanks, "ep: 4 buffers per rank, 2..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < W, "ep: bad rank");
  EpParams p{};
  for (int q = 0; q < W; ++q) {
    TORCH_CHECK((bufs[4 * q] | bufs[4 * q + 1] | bufs[4 * q + 2] | bufs[4 * q + 3]) % 16 == 0,
                "ep: 16B alignment");
    p.recv_x_peer[q] = reinterpret_cast<__nv_bfloat16*>(bufs[4 * q]);
    p.recv_meta_peer[q] = reinterpret_cast<int*>(bufs[4 * q + 1]);
    p.back_y_peer[q] = reinterpret_cast<__nv_bfloat16*>(bufs[4 * q + 2]);
    p.pad_peer[q] = reinterpret_cast<uint32_t*>(bufs[4 * q + 3]);
  }
  p.recv_x_local = p.recv_x_peer[rank];
  p.recv_meta_local = p.recv_meta_peer[rank];
  p.back_y_local = p.back_y_peer[rank];
  p.pad_local = p.pad_peer[rank];
  p.rank = (int)rank;
  p.world = W;
  p.H = (int)H;
  p.k = (int)k;
  p.E_local = (int)E_local;
  p.T_cap = (int)T_cap;
  p.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
  p.err = device_status_ptr(device);
  return p;
}

void ep_dispatch(const std::vector<int64_t>& bufs, int64_t rank, int64_t E_local, int64_t T_cap,
                 int64_t timeout_ms, const at::Tensor& x, const at::Tensor& ids,
                 const at::Tensor& w, at::Tensor& slot, at::Tensor& send_count) {
  CHECK_CUDA(x); CHECK_BF16(x);
  TORCH_CHECK(x.is_contiguous() && ids.is_contiguous() && w.is_contiguous(), "ep_dispatch: contiguous");
  TORCH_CHECK(ids.scalar_type() == at::kInt && w.scalar_type() == at::kFloat &&
                  slot.scalar_type() == at::kInt && send_count.scalar_type() == at::kInt,
              "ep_dispatch: dtypes");
  const int T = (int)x.size(0), k = (int)ids.size(1);
  const EpParams p = make_ep(bufs, rank, x.size(1), k, E_local, T_cap, timeout_ms, x.get_device());
  TORCH_CHECK(slot.numel() >= (int64_t)T * p.world && send_count.numel() >= p.world, "ep_dispatch: scratch");
  c10::cuda::CUDAGuard g(x.device());
  ep_dispatch_launch(p, x.data_ptr(), ids.data_ptr<int>(), w.data_ptr<float>(), T,
                     slot.data_ptr<int>(), send_count.data_ptr<int>(), cur_stream());
}

void ep_receive(const std::vector<int64_t>& bufs, int64_t rank, int64_t E_local, int64_t T_cap,
                int64_t timeout_ms, at::Tensor& xc, at::Tensor& idc, at::Tensor& wc,
                at::Tensor& row_src, at::Tensor& n_rows) {
  CHECK_BF16(xc);
  const int n_max = (int)xc.size(0), k = (int)idc.size(1);
  TORCH_CHECK(idc.size(0) >= n_max && wc.size(0) >= n_max && row_src.numel() >= n_max,
              "ep_receive: buffers");
  const EpParams p = make_ep(bufs, rank, xc.size(1), k, E_local, T_cap, timeout_ms, xc.get_device());
  c10::cuda::CUDAGuard g(xc.device());
  ep_receive_launch(p, xc.data_ptr(), idc.data_ptr<int>(), wc.data_ptr<float>(),
                    row_src.data_ptr<int>(), n_rows.data_ptr<int>(), n_max, cur_stream());
}

void ep_return(const std::vector<int64_t>& bufs, int64_t rank, int64_t E_local, int64_t T_cap,
               int64_t timeout_ms, int64_t k, const at::Tensor& y, const at::Tensor& row_src,
               const at::Tensor& n_rows) {
  CHECK_BF16(y);
  const EpParams p = make_ep(bufs, rank, y.size(1), k, E_local, T_cap, timeout_ms, y.get_device());
  c10::cuda::CUDAGuard g(y.device());
  ep_return_launch(p, y.data_ptr(), row_src.data_ptr<int>(), n_rows.data_ptr<int>(),
                   (int)y.size(0), cur_stream());
}

void ep_finish(const std::vector<int64_t>& bufs, int64_t rank, int64_t E_local, int64_t T_cap,
               int64_t timeout_ms, int64_t k, const at::Tensor& slot,
               const c10::optional<at::Tensor>& shared, at::Tensor& out) {
  CHECK_BF16(out);
  TORCH_CHECK(out.is_contiguous(), "ep_finish: out contiguous");
  if (shared) TORCH_CHECK(shared->is_contiguous() && shared->sizes() == out.sizes(), "ep_finish: shared");
  const EpParams p = make_ep(bufs, rank, out.size(1), k, E_local, T_cap, timeout_ms, out.get_device());
  c10::cuda::CUDAGuard g(out.device());
  ep_finish_launch(p, slot.data_ptr<int>(), (int)out.size(0),
                   shared ? shared->data_ptr() : nullptr, out.data_ptr(), cur_stream());
}

// All-gather -> GEMM: out [T, N] = concat over ranks of shard [T/W, K] (rank
// order) times w [N, K]^T, the gather done inside the GEMM through the
// symmetric buffers xfull (each [2][t_max][K] bf16) and pads (16 words).
void gemm_ag(const at::Tensor& w, at::Tensor& out, const at::Tensor& shard,
             const std::vector<int64_t>& xfull_ptrs, const std::vector<int64_t>& pad_ptrs,
             int64_t rank, int64_t t_max, int64_t cfg, int64_t splits, int64_t timeout_ms) {
  const int W = (int)xfull_ptrs.size();
  TORCH_CHECK(W >= 2 && W <= kMaxRanks && (int)pad_ptrs.size() == W, "gemm_ag: 2..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < W, "gemm_ag: bad rank");
  CHECK_CUDA(shard); CHECK_BF16(shard); CHECK_BF16(w); CHECK_BF16(out);
  TORCH_CHECK(shard.dim() == 2 && shard.is_contiguous() && w.dim() == 2 && w.stride(1) == 1 &&
              w.size(1) == shard.size(1), "gemm_ag: shard [T/W, K] contiguous, w [N, K]");
  const int64_t rpr = shard.size(0), K = shard.size(1), T = rpr * W, N = w.size(0);
  TORCH_CHECK(out.dim() == 2 && out.size(0) == T && out.size(1) == N && out.stride(1) == 1,
              "gemm_ag: out [T, N]");
  TORCH_CHECK(T <= t_max && K % 8 == 0 && (reinterpret_cast<uintptr_t>(shard.data_ptr()) & 15) == 0,
              "gemm_ag: T <= t_max, K % 8, 16B-aligned shard");
  AgParams ag{};
  for (int q = 0; q < W; ++q) {
    TORCH_CHECK(xfull_ptrs[q] % 16 == 0 && pad_ptrs[q] % 16 == 0, "gemm_ag: 16B alignment");
    ag.xfull_peer[q] = reinterpret_cast<uint8_t*>(xfull_ptrs[q]);
    ag.pad_peer[q] = reinterpret_cast<uint32_t*>(pad_ptrs[q]);
  }
  ag.pad_local = ag.pad_peer[rank];
  ag.shard = shard.data_ptr();
  ag.rank = (int)rank;
  ag.world = W;
  ag.rows_per_rank = (int)rpr;
  ag.t_max = (int)t_max;
  ag.K = (int)K;
  ag.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
  unsigned int* err = device_status_ptr(shard.get_device());
  c10::cuda::CUDAGuard g(shard.device());
  gemm_ag_launch(w.data_ptr(), out.data_ptr(), (int)T, (int)N, (int)K, (int)w.stride(0),
                 (int)out.stride(0), (int)cfg, (int)splits, ag, err, cur_stream());
}

// Vocab-parallel sampler exchange over peer memory. bufs = [recv, pad] per
// rank. mode 0: src0 = values [rows] fp32, src1 = ids [rows] int32 ->
// out0 = merged ids [rows] int32. mode 1: src0 / src1 = values / ids
// [rows, C] -> out0 = values [rows, W*C] fp32, out1 = ids [rows, W*C] int32.
void tp_exchange(const std::vector<int64_t>& bufs, int64_t rank, int64_t cap, int64_t mode,
                 const at::Tensor& src0, const at::Tensor& src1, at::Tensor& out0,
                 const c10::optional<at::Tensor>& out1, int64_t timeout_ms) {
  const int W = (int)bufs.size() / 2;
  TORCH_CHECK((int)bufs.size() == 2 * W && (W == 2 || W == 4 || W == 8),
              "tp_exchange: [recv, pad] per rank, 2, 4 or 8 ranks");
  TORCH_CHECK(rank >= 0 && rank < W, "tp_exchange: bad rank");
  CHECK_CUDA(src0); CHECK_CUDA(src1); CHECK_CUDA(out0);
  TORCH_CHECK(src0.is_contiguous() && src1.is_contiguous() && out0.is_contiguous(),
              "tp_exchange: contiguous tensors");
  TORCH_CHECK(src0.scalar_type() == at::kFloat && src1.scalar_type() == at::kInt,
              "tp_exchange: src0 fp32 values, src1 int32 ids");
  TORCH_CHECK(src0.sizes() == src1.sizes(), "tp_exchange: values / ids shapes differ");
  TpExchangeParams p{};
  for (int q = 0; q < W; ++q) {
    TORCH_CHECK(bufs[2 * q] % 16 == 0 && bufs[2 * q + 1] % 16 == 0, "tp_exchange: 16B alignment");
    p.recv_peer[q] = reinterpret_cast<uint8_t*>(bufs[2 * q]);
    p.pad_peer[q] = reinterpret_cast<uint32_t*>(bufs[2 * q + 1]);
  }
  p.recv_local = p.recv_peer[rank];
  p.pad_local = p.pad_peer[rank];
  p.rank = (int)rank;
  p.world = W;
  p.mode = (int)mode;
  p.cap = cap;
  p.src0 = src0.data_ptr();
  p.n0 = src0.numel() * 4;
  p.src1 = src1.data_ptr();
  p.n1 = src1.numel() * 4;
  if (mode == kTpXchgTop1) {
    TORCH_CHECK(src0.dim() == 1 && out0.scalar_type() == at::kInt && out0.numel() == src0.numel(),
                "tp_exchange top1: values / ids [rows], out int32 [rows]");
    p.rows = (int)src0.numel();
    p.C = 1;
    p.out_ids = out0.data_ptr<int>();
  } else {
    TORCH_CHECK(mode == kTpXchgGather, "tp_exchange: mode 0 (top-1) or 1 (gather)");
    TORCH_CHECK(src0.dim() == 2 && out1.has_value(), "tp_exchange gather: [rows, C] and two outputs");
    p.rows = (int)src0.size(0);
    p.C = (int)src0.size(1);
    TORCH_CHECK(out0.scalar_type() == at::kFloat && out0.numel() == (int64_t)W * src0.numel() &&
                out1->scalar_type() == at::kInt && out1->numel() == out0.numel() &&
                out1->is_contiguous(), "tp_exchange gather: outputs [rows, W*C] fp32 / int32");
    p.out_v = out0.data_ptr<float>();
    p.out_i = out1->data_ptr<int>();
  }
  p.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
  p.err = device_status_ptr(out0.get_device());
  c10::cuda::CUDAGuard g(out0.device());
  tp_exchange_launch(p, cur_stream());
}

// Row-parallel GEMM x @ lin_w^T into this rank's stage, fused in one kernel
// with the all-reduce + residual add + RMSNorm. Returns false when the
// shape / tile is not taken (nothing launched; the caller runs the unfused pair).
bool gemm_ar_rmsnorm(const at::Tensor& x, const at::Tensor& lin_w,
                     const std::vector<int64_t>& stage_ptrs, const std::vector<int64_t>& res_ptrs,
                     const std::vector<int64_t>& out_ptrs, const std::vector<int64_t>& flag_ptrs,
                     int64_t rank, const at::Tensor& w, double eps, int64_t timeout_ms,
                     int64_t cfg, int64_t splits,
                     const std::vector<int64_t>& mc_ptrs) {
  const int W = (int)stage_ptrs.size();
  TORCH_CHECK(W == 1 || W == 2 || W == 4 || W == 8,
              "gemm_ar_rmsnorm: world size must be 1 (TP1: add + RMSNorm), 2, 4 or 8");
  TORCH_CHECK((int)res_ptrs.size() == W && (int)out_ptrs.size() == W && (int)flag_ptrs.size() == W,
              "gemm_ar_rmsnorm: pointer lists must have one entry per rank");
  TORCH_CHECK(rank >= 0 && rank < W, "gemm_ar_rmsnorm: bad rank");
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(lin_w); CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && lin_w.dim() == 2 && x.stride(1) == 1 && lin_w.stride(1) == 1 &&
              x.size(1) == lin_w.size(1), "gemm_ar_rmsnorm: x [T, K], lin_w [H, K]");
  const int64_t T = x.size(0), H = lin_w.size(0), K = x.size(1);
  TORCH_CHECK(w.numel() == H && H % 8 == 0, "gemm_ar_rmsnorm: norm weight size / H % 8");
  ArRmsNormParams p{};
  for (int q = 0; q < W; ++q) {
    p.stage_peer[q] = reinterpret_cast<const __nv_bfloat16*>(stage_ptrs[q]);
    p.res_peer[q] = reinterpret_cast<__nv_bfloat16*>(res_ptrs[q]);
    p.out_peer[q] = reinterpret_cast<__nv_bfloat16*>(out_ptrs[q]);
    p.flags_peer[q] = reinterpret_cast<uint32_t*>(flag_ptrs[q]);
    TORCH_CHECK((stage_ptrs[q] | res_ptrs[q] | out_ptrs[q]) % 16 == 0,
                "gemm_ar_rmsnorm: 16B alignment");
  }
  p.flags_local = p.flags_peer[rank];
  p.res_local = p.res_peer[rank];
  p.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.rank = (int)rank;
  p.world = W;
  p.T = (int)T;
  p.H = (int)H;
  p.eps = (float)eps;
  p.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
  p.err = device_status_ptr(x.get_device());
  set_mc(p, mc_ptrs);
  c10::cuda::CUDAGuard g(x.device());
  return gemm_ar_rmsnorm_launch(x.data_ptr(), lin_w.data_ptr(), (int)T, (int)H, (int)K,
                                (int)x.stride(0), (int)lin_w.stride(0), (int)cfg, (int)splits, p,
                                p.err, cur_stream());
}

void argmax(at::Tensor& ids, const c10::optional<at::Tensor>& vals, const at::Tensor& logits,
            int64_t id_offset) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "argmax: 2-D logits");
  TORCH_CHECK(ids.scalar_type() == at::kInt, "argmax: ids int32");
  const bool bf = logits.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf || logits.scalar_type() == at::kFloat, "argmax: bf16 or fp32 logits");
  c10::cuda::CUDAGuard g(logits.device());
  argmax_launch(logits.data_ptr(), bf, (int)logits.size(0), (int)logits.size(1),
                (int)logits.stride(0), ids.data_ptr<int>(),
                vals ? vals->data_ptr<float>() : nullptr, (int)id_offset, cur_stream());
}

void silu_mul(at::Tensor& out, const at::Tensor& x, int64_t block,
              const c10::optional<at::Tensor>& n_rows) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(out);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1, "silu_mul: 2-D rows");
  if (n_rows) TORCH_CHECK(n_rows->scalar_type() == at::kInt, "silu_mul: n_rows int32");
  c10::cuda::CUDAGuard g(x.device());
  silu_mul_launch(out.data_ptr(), x.data_ptr(), (int)x.size(0), (int)(x.size(1) / 2),
                  (int)x.stride(0), (int)out.stride(0), cur_stream(), (int)block,
                  n_rows ? n_rows->data_ptr<int>() : nullptr);
}

void embedding(at::Tensor& out, const at::Tensor& ids, const at::Tensor& table,
               int64_t vocab_start) {
  CHECK_CUDA(ids); CHECK_BF16(table); CHECK_BF16(out);
  TORCH_CHECK(ids.scalar_type() == at::kLong, "embedding: ids int64");
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous(), "embedding: contiguous");
  c10::cuda::CUDAGuard g(ids.device());
  embedding_launch(out.data_ptr(), ids.data_ptr<int64_t>(), table.data_ptr(), (int)ids.numel(),
                   (int)table.size(1), vocab_start, vocab_start + table.size(0), cur_stream());
}

}  // namespace
}  // namespace b200

TORCH_LIBRARY(_b200_C, m) {
  m.def("abi_version() -> int", &b200::abi_version);
  m.def("init_device(int device) -> ()", &b200::init_device);
  m.def("read_status(int device, bool clear) -> int", &b200::read_status);
  m.def("gemm_bf16(Tensor a, Tensor w, int cfg=-1) -> Tensor");
  m.def("gemm_bf16_out(Tensor(a!) out, Tensor a, Tensor w, int cfg=-1, int splits=0) -> ()");
  m.def("gemm_configure_workspace(int device, int ws_bytes, int n_counters) -> ()",
        &b200::gemm_configure_workspace_op);
  m.def("gemm_bf16_plan(int M, int N, int K, int epi, int num_sm) -> int[]",
        &b200::gemm_bf16_plan_op);
  m.def("gemm_set_plan(int M, int N, int K, int epi, int cfg, int splits) -> ()",
        &b200::gemm_set_plan_op);
  m.def("gemm_clear_plans() -> ()", &b200::gemm_clear_plans_op);
  m.def("gemm_set_timeline(Tensor? buf) -> ()", &b200::gemm_set_timeline_op);
  m.def("attn_fa_set_timeline(Tensor? buf) -> ()", &b200::attn_fa_set_timeline_op);
  m.def("gemm_export_plans() -> int[]", &b200::gemm_export_plans_op);
  m.def("gemm_bf16_silu_mul_out(Tensor(a!) out, Tensor a, Tensor w, int cfg=-1) -> ()");
  m.def("gemm_bf16_config(int M, int N, int K, int epi) -> int", &b200::gemm_bf16_config);
  m.def("gemm_wq_out(Tensor(a!) out, Tensor a, Tensor w_raw, int fmt, Tensor scales, "
        "float out_scale, int bn=0, int splits=0) -> ()");
  m.def("dequant_weight(Tensor(a!) out, Tensor w_raw, int fmt, Tensor scales) -> ()");
  m.def("moe_topk(Tensor(a!) w, Tensor(b!) ids, Tensor logits, int k, bool use_sigmoid, bool renorm, "
        "Tensor? bias) -> ()");
  m.def("moe_router(Tensor(a!) w, Tensor(b!) ids, Tensor x, Tensor wr, int k, bool use_sigmoid, "
        "bool renorm, Tensor? bias, Tensor(c!) logits, Tensor(d!) tile_ctr) -> ()");
  m.def("moe_permute(Tensor ids, int E, int e_base, Tensor? x, Tensor(a!)? x_perm, Tensor(b!) counts, "
        "Tensor(c!) offsets, Tensor(d!) rank_scratch, Tensor(e!) pos, Tensor(f!) src_row, "
        "int align=1) -> ()");
  m.def("quant_nvfp4_act(Tensor x, Tensor(a!) xq, Tensor(b!) sf, Tensor(c!) rs, "
        "Tensor? n_rows=None) -> ()");
  m.def("gemm_nvfp4_out(Tensor(a!) out, Tensor xq, Tensor sfa, Tensor rs, Tensor wq, Tensor sfw, "
        "float g, int swap=-1) -> ()");
  m.def("gemm_nvfp4_grouped_out(Tensor(a!) out, Tensor xq, Tensor sfx, Tensor rs, Tensor w_stk, "
        "Tensor sfw, float g, int E, int N, Tensor row_off, Tensor(b!) tile_off) -> ()");
  m.def("moe_combine(Tensor(a!) out, Tensor y, Tensor pos, Tensor w, Tensor? shared, float shared_scale) -> ()");
  m.def("gemm_grouped_out(Tensor(a!) out, Tensor x, Tensor w_stk, int E, int N, Tensor row_off, "
        "Tensor(b!) tile_off, int fmt, Tensor? scales, float out_scale, int bn=0) -> ()");
  m.def("quant_fp8_act(Tensor x, Tensor(a!) xq, Tensor(b!) sa) -> ()");
  m.def("gemm_fp8_out(Tensor(a!) out, Tensor xq, Tensor sa, Tensor wq, Tensor sw, int bn=0) -> ()");
  m.def("gemm_fp8_grouped_out(Tensor(a!) out, Tensor xq, Tensor sa, Tensor w_stk, Tensor sw, "
        "int E, int N, Tensor row_off, Tensor(b!) tile_off, int bn=0) -> ()");
  m.def("gumbel_argmax(Tensor(a!) ids, Tensor(b!) vals, Tensor logits, Tensor temperature, "
        "Tensor seeds, int offset, int id_offset, Tensor? row_offsets=None) -> ()");
  m.def("topk_candidates(Tensor(a!) vals, Tensor(b!) ids, Tensor logits, int K, int id_offset) -> ()");
  m.def("sample_candidates(Tensor(a!) out, Tensor cand_v, Tensor cand_i, Tensor temperature, "
        "Tensor top_k, Tensor top_p, Tensor seeds, int offset) -> ()");
  m.def("causal_conv1d(Tensor(a!) y, Tensor x, Tensor w, Tensor? bias, Tensor(b!) state, "
        "Tensor cu, Tensor slots, bool silu, bool write_state=True) -> ()");
  m.def("gdn_recurrent(Tensor(a!) o, Tensor q, Tensor k, Tensor v, Tensor a, Tensor b, "
        "Tensor A_log, Tensor dt_bias, Tensor(b!) state, Tensor cu, Tensor slots, int HK, int HV, "
        "bool reset_state, bool write_state=True, bool chunked=False, Tensor? has_init=None) -> ()");
  m.def("gated_rmsnorm(Tensor(a!) o, Tensor z, Tensor w, int H, float eps) -> ()");
  m.def("rejection_sample(Tensor(a!) out_tokens, Tensor(b!) num_out, Tensor target_logits, "
        "Tensor draft_logits, Tensor draft_ids, Tensor temperature, Tensor seeds, int offset) -> ()");
  m.def("rms_norm(Tensor(a!) out, Tensor x, Tensor w, float eps) -> ()");
  m.def("fused_add_rms_norm(Tensor(a!) x, Tensor(b!) residual, Tensor w, float eps) -> ()");
  m.def(
      "rope_kv_write(Tensor(a!) qkv, Tensor positions, Tensor cos_sin, Tensor(b!) k_cache, "
      "Tensor(c!) v_cache, Tensor slot_mapping, int num_q_heads, int num_kv_heads, "
      "Tensor? q_norm, Tensor? k_norm, float eps) -> ()");
  m.def(
      "paged_attention(Tensor(a!) out, Tensor q, Tensor k_cache, Tensor v_cache, "
      "Tensor block_table, Tensor seq_lens, Tensor cu_q, int max_q_len, float scale, int window, "
      "Tensor? sinks, bool decode, int num_splits, Tensor? part_o, Tensor? part_ml) -> ()");
  m.def("ep_dispatch(int[] bufs, int rank, int E_local, int T_cap, int timeout_ms, Tensor x, "
        "Tensor ids, Tensor w, Tensor(a!) slot, Tensor(b!) send_count) -> ()");
  m.def("ep_receive(int[] bufs, int rank, int E_local, int T_cap, int timeout_ms, Tensor(a!) xc, "
        "Tensor(b!) idc, Tensor(c!) wc, Tensor(d!) row_src, Tensor(e!) n_rows) -> ()");
  m.def("ep_return(int[] bufs, int rank, int E_local, int T_cap, int timeout_ms, int k, Tensor y, "
        "Tensor row_src, Tensor n_rows) -> ()");
  m.def("gemm_ag(Tensor w, Tensor(a!) out, Tensor shard, int[] xfull_ptrs, int[] pad_ptrs, "
        "int rank, int t_max, int cfg=-1, int splits=0, int timeout_ms=2000) -> ()");
  m.def("tp_exchange(int[] bufs, int rank, int cap, int mode, Tensor src0, Tensor src1, "
        "Tensor(a!) out0, Tensor(b!)? out1, int timeout_ms) -> ()");
  m.def("ep_finish(int[] bufs, int rank, int E_local, int T_cap, int timeout_ms, int k, "
        "Tensor slot, Tensor? shared, Tensor(a!) out) -> ()");
  m.def("ar_rmsnorm(int[] stage_ptrs, int[] res_ptrs, int[] out_ptrs, int[] flag_ptrs, int rank, "
        "int T, int H, Tensor w, float eps, int timeout_ms, int grid, int[] mc_ptrs=[]) -> ()");
  m.def("gemm_ar_rmsnorm(Tensor x, Tensor lin_w, int[] stage_ptrs, int[] res_ptrs, int[] out_ptrs, "
        "int[] flag_ptrs, int rank, Tensor w, float eps, int timeout_ms, int cfg, int splits, "
        "int[] mc_ptrs=[]) -> bool");
  m.def("kv_cache_write(Tensor k, Tensor v, Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor slots) -> ()");
  m.def("argmax(Tensor(a!) ids, Tensor(b!)? vals, Tensor logits, int id_offset) -> ()");
  m.def("silu_mul(Tensor(a!) out, Tensor x, int block=0, Tensor? n_rows=None) -> ()");
  m.def("embedding(Tensor(a!) out, Tensor ids, Tensor table, int vocab_start) -> ()");
}

TORCH_LIBRARY_IMPL(_b200_C, CUDA, m) {
  m.impl("gemm_bf16", &b200::gemm_bf16);
  m.impl("gemm_bf16_out", &b200::gemm_bf16_out);
  m.impl("gemm_bf16_silu_mul_out", &b200::gemm_bf16_silu_mul_out);
  m.impl("rms_norm", &b200::rms_norm);
  m.impl("rejection_sample", &b200::rejection_sample);
  m.impl("causal_conv1d", &b200::causal_conv1d);
  m.impl("gdn_recurrent", &b200::gdn_recurrent);
  m.impl("gated_rmsnorm", &b200::gated_rmsnorm);
  m.impl("gumbel_argmax", &b200::gumbel_argmax);
  m.impl("topk_candidates", &b200::topk_candidates);
  m.impl("sample_candidates", &b200::sample_candidates);
  m.impl("moe_topk", &b200::moe_topk);
  m.impl("moe_router", &b200::moe_router);
  m.impl("moe_permute", &b200::moe_permute);
  m.impl("moe_combine", &b200::moe_combine);
  m.impl("gemm_grouped_out", &b200::gemm_grouped_out);
  m.impl("gemm_wq_out", &b200::gemm_wq_out);
  m.impl("quant_fp8_act", &b200::quant_fp8_act);
  m.impl("quant_nvfp4_act", &b200::quant_nvfp4_act);
  m.impl("gemm_nvfp4_out", &b200::gemm_nvfp4_out);
  m.impl("gemm_nvfp4_grouped_out", &b200::gemm_nvfp4_grouped_out);
  m.impl("ep_dispatch", &b200::ep_dispatch);
  m.impl("ep_receive", &b200::ep_receive);
  m.impl("ep_return", &b200::ep_return);
  m.impl("ep_finish", &b200::ep_finish);
  m.impl("tp_exchange", &b200::tp_exchange);
  m.impl("gemm_ag", &b200::gemm_ag);
  m.impl("gemm_fp8_out", &b200::gemm_fp8_out);
  m.impl("gemm_fp8_grouped_out", &b200::gemm_fp8_grouped_out);
  m.impl("dequant_weight", &b200::dequant_weight);
  m.impl("fused_add_rms_norm", &b200::fused_add_rms_norm);
  m.impl("rope_kv_write", &b200::rope_kv_write);
  m.impl("paged_attention", &b200::paged_attention);
  m.impl("argmax", &b200::argmax);
  m.impl("kv_cache_write", &b200::kv_cache_write);
  m.impl("ar_rmsnorm", &b200::ar_rmsnorm);
  m.impl("gemm_ar_rmsnorm", &b200::gemm_ar_rmsnorm);
  m.impl("silu_mul", &b200::silu_mul);
  m.impl("embedding", &b200::embedding);
}
