"""Quantised linear layers: block-FP8 (W8A8 on kind::f8f6f4 tensor cores, or
W8A16), AWQ int4 (W4A16), NVFP4 (W4A16), on the tcgen05 GEMMs.

Block-FP8 runs W8A8 by default (``VLLM_B200_FP8_W8A8``): activations are
quantised per token and 128-wide K group to e4m3 (fp32 scale = group amax /
448), the GEMM multiplies e4m3 x e4m3 on the tensor cores and promotes each
128-wide K block's partial sum into fp32 with both scales. The weight-only
formats dequantise in the GEMM producer (decode shapes, M <= 256) or
dequantise then run the bf16 GEMM (prefill).

Checkpoint formats (HF safetensors) and the in-memory layouts:

* FP8 (``quant_method: fp8``, ``weight_block_size: [128, 128]``): ``weight``
  e4m3 ``[N, K]`` + ``weight_scale_inv`` fp32 ``[ceil(N/128), ceil(K/128)]``
  (the dequant multiplier). Kept as is.
* AWQ (GEMM version, group 128): ``qweight`` int32 ``[K, N/8]``, ``qzeros``
  int32 ``[K/128, N/8]``, ``scales`` fp16 ``[K/128, N]``, nibbles packed in
  the AWQ column order [0, 2, 4, 6, 1, 3, 5, 7]. Repacked at load time to
  row-major int4 ``[N, K/2]`` (low nibble = even k) + bf16 ``(s, -z*s)`` pairs
  ``[N, 2*K/128]``, so the kernel dequantises with one FMA.
* NVFP4 (ModelOpt): ``weight`` uint8 ``[N, K/2]`` (two e2m1, low nibble =
  even k), ``weight_scale`` e4m3 ``[N, K/16]``, ``weight_scale_2`` fp32 global.
  Kept as is; the global scale multiplies the GEMM output.

Reference parity: ``Fp8Sm70LinearMethod`` (``sm70/vllm_sm70/quant/fp8_linear.py``),
``ModelOptNvFp4Sm70LinearMethod`` (``quant/nvfp4_linear.py``), AWQ ops
(``csrc/turbomind/ops/tm_awq_sm70.cu``); their dequantisers
(``sm70/tests/ops/_ref.py:1-49``: ``nvfp4_dequant``, ``fp8_block_dequant``).
"""
from __future__ import annotations

import torch

from .. import _ext, envs
from ..models.layers import Linear
from ..utils import launch_count
from . import linear as _lin

FMT_ID = {"fp8": 1, "awq": 2, "nvfp4": 3}
E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])
AWQ_ORDER = [0, 2, 4, 6, 1, 3, 5, 7]
AWQ_INV = [0, 4, 1, 5, 2, 6, 3, 7]
FP8_MAX = 448.0
WQ_MAX_M = 256


# ------------------------------------------------------------------ quantisers
def quantize_fp8_block(w: torch.Tensor, block: int = 128):
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    wp = torch.zeros(nb * block, kb * block, device=w.device, dtype=torch.float32)
    wp[:N, :K] = w.float()
    blocks = wp.view(nb, block, kb, block)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / FP8_MAX
    q = (blocks / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX)
    q = q.view(nb * block, kb * block)[:N, :K].to(torch.float8_e4m3fn)
    return q.contiguous(), scale.contiguous()


def quantize_awq(w: torch.Tensor, group: int = 128):
    """Asymmetric int4 per (row, group). Returns AutoAWQ-layout tensors."""
    N, K = w.shape
    g = w.float().view(N, K // group, group)
    mn, mx = g.amin(-1), g.amax(-1)
    scale = ((mx - mn) / 15.0).clamp_min(1e-8)
    zero = torch.round(-mn / scale).clamp(0, 15)
    q = torch.clamp(torch.round(g / scale[..., None]) + zero[..., None], 0, 15).to(torch.int32)
    q = q.view(N, K)
    # AutoAWQ GEMM layout: qweight [K, N/8], column j of pack c is nibble AWQ_INV[j].
    qt = q.t().contiguous().view(K, N // 8, 8)
    qweight = torch.zeros(K, N // 8, dtype=torch.int32, device=w.device)
    for i in range(8):
        qweight |= (qt[:, :, AWQ_ORDER[i]] & 0xF) << (4 * i)
    zt = zero.to(torch.int32).t().contiguous().view(K // group, N // 8, 8)
    qzeros = torch.zeros(K // group, N // 8, dtype=torch.int32, device=w.device)
    for i in range(8):
        qzeros |= (zt[:, :, AWQ_ORDER[i]] & 0xF) << (4 * i)
    return qweight, qzeros, scale.t().contiguous().to(torch.float16)


def unpack_awq(packed: torch.Tensor) -> torch.Tensor:
    """int32 [R, C/8] in AWQ order -> int32 [R, C] nibble values."""
    R, C8 = packed.shape
    out = torch.empty(R, C8, 8, dtype=torch.int32, device=packed.device)
    for i in range(8):
        out[:, :, AWQ_ORDER[i]] = (packed >> (4 * i)) & 0xF
    return out.view(R, C8 * 8)


def quantize_nvfp4(w: torch.Tensor, block: int = 16):
    N, K = w.shape
    wf = w.float()
    gmax = wf.abs().max().clamp_min(1e-12)
    gscale = gmax / (FP8_MAX * 6.0)
    blocks = wf.view(N, K // block, block)
    bmax = blocks.abs().amax(-1)
    bscale = (bmax / 6.0 / gscale).clamp(max=FP8_MAX).to(torch.float8_e4m3fn)
    eff = bscale.float() * gscale
    x = blocks / eff.clamp_min(1e-12)[..., None]
    mags = E2M1[:8].to(w.device)
    idx = (x.abs()[..., None] - mags).abs().argmin(-1)
    code = idx | ((x < 0).to(torch.int64) << 3)
    code = code.view(N, K).to(torch.uint8)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).contiguous()
    return packed, bscale.contiguous(), float(gscale)


def w8a8_enabled() -> bool:
    return bool(envs.get("VLLM_B200_FP8_W8A8"))


def quant_fp8_act_ref(x: torch.Tensor):
    """CPU/GPU torch oracle of the activation quantiser: per row and 128-wide K
    group, scale = amax / 448 (1 for an all-zero group), q = e4m3(x * 448 / amax)
    rounded to nearest even after clamping to +-448. Returns (q [M, K] e4m3,
    scale [M, ceil(K/128)] fp32) -- the same values the CUDA kernel writes."""
    xf = x.float()
    M, K = xf.shape
    G = (K + 127) // 128
    xp = torch.zeros(M, G * 128, dtype=torch.float32, device=xf.device)
    xp[:, :K] = xf
    g = xp.view(M, G, 128)
    amax = g.abs().amax(-1)
    pos = amax > 0
    one = torch.ones_like(amax)
    # Tensor / tensor: an IEEE division (a python-scalar divisor may be turned
    # into a multiplication by its reciprocal, which rounds differently).
    fmax = torch.full_like(amax, FP8_MAX)
    scale = torch.where(pos, amax / fmax, one)
    inv = torch.where(pos, fmax / torch.where(pos, amax, one), one)
    q = (g * inv[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(M, G * 128)[:, :K].contiguous(), scale


def fp8_act_dequant_ref(x: torch.Tensor) -> torch.Tensor:
    """fp32 value of x after the W8A8 activation quantisation round trip."""
    q, s = quant_fp8_act_ref(x)
    return q.float() * s.repeat_interleave(128, 1)[:, : q.shape[1]]


def quant_fp8_act(x: torch.Tensor):
    """(xq uint8 [M, K] e4m3 bytes, sa fp32 [ceil(K/128), M']) on the CUDA kernel."""
    M, K = x.shape
    xq = torch.empty(M, K, dtype=torch.uint8, device=x.device)
    sa = torch.empty((K + 127) // 128, max(4, (M + 3) // 4 * 4), dtype=torch.float32,
                     device=x.device)
    torch.ops._b200_C.quant_fp8_act(x, xq, sa)
    launch_count.add(1)
    return xq, sa


def gemm_fp8(x: torch.Tensor, w_raw: torch.Tensor, sw: torch.Tensor,
             out: torch.Tensor | None = None, bn: int = 0) -> torch.Tensor:
    """W8A8 block-FP8 GEMM: ``x [M, K] bf16`` quantised on the fly, times the
    e4m3 weight ``w_raw [N, K]`` with block scales ``sw [ceil(N/128), ceil(K/128)]``."""
    if out is None:
        out = torch.empty(x.shape[0], w_raw.shape[0], dtype=torch.bfloat16, device=x.device)
    xq, sa = quant_fp8_act(x)
    torch.ops._b200_C.gemm_fp8_out(out, xq, sa, w_raw, sw, bn)
    launch_count.add(1)
    return out


# ------------------------------------------------------------------ NVFP4 W4A4
def w4a4_enabled() -> bool:
    return bool(envs.get("VLLM_B200_NVFP4_W4A4"))


def nvfp4_sf_atoms(sf: torch.Tensor) -> torch.Tensor:
    """Block scales ``[N, K/16]`` (e4m3 bytes, row-major) -> the tensor-core
    atom order ``[ceil(N/128)][K/64][512]``: row r's 4 scales of 64-k group
    kg at byte (r % 32) * 16 + ((r % 128) / 32) * 4 + j. Padded rows get 0."""
    N, G = sf.shape
    assert G % 4 == 0, "K must be a multiple of 64"
    Np = (N + 127) // 128 * 128
    s = torch.zeros(Np, G, dtype=torch.uint8, device=sf.device)
    s[:N] = sf.view(torch.uint8)
    # [nb, m1, m0, kg, j] -> [nb, kg, m0, m1, j]
    s = s.view(Np // 128, 4, 32, G // 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return s.view(-1)


def _e2m1_round(y: torch.Tensor) -> torch.Tensor:
    """Round to the nearest e2m1 value (ties to the even mantissa), saturating
    at +-6: the rounding of ``cvt.rn.satfinite.e2m1x2.f32``."""
    a = y.abs()
    r = torch.where(a <= 0.25, 0.0,
        torch.where(a < 0.75, 0.5,
        torch.where(a <= 1.25, 1.0,
        torch.where(a < 1.75, 1.5,
        torch.where(a <= 2.5, 2.0,
        torch.where(a < 3.5, 3.0,
        torch.where(a <= 5.0, 4.0, 6.0)))))))
    return torch.copysign(r, y)


def quant_nvfp4_act_ref(x: torch.Tensor):
    """Torch oracle of the W4A4 activation quantiser: per row rs = amax / 2688
    (448 * 6; 1 for a zero row), per 16-element block s = e4m3(amax_blk / 6 /
    rs), values e2m1(x / (s * rs)). Returns (e2m1 values [M, K] fp32, block
    scales [M, K/16] as fp32 of the e4m3 bytes, rs [M])."""
    xf = x.float()
    M, K = xf.shape
    amax = xf.abs().amax(1)
    one = torch.ones_like(amax)
    rs = torch.where(amax > 0, amax / torch.full_like(amax, 2688.0), one)
    blocks = xf.view(M, K // 16, 16)
    bmax = blocks.abs().amax(-1)
    s = (bmax / torch.full_like(bmax, 6.0)) / rs[:, None]
    s8 = s.clamp(max=FP8_MAX).to(torch.float8_e4m3fn)
    sdec = s8.float() * rs[:, None]
    inv = torch.where(sdec > 0, torch.ones_like(sdec) / torch.where(sdec > 0, sdec, 1.0), 0.0)
    q = _e2m1_round(blocks * inv[..., None]).view(M, K)
    return q, s8.float(), rs


def nvfp4_act_dequant_ref(x: torch.Tensor) -> torch.Tensor:
    q, s, rs = quant_nvfp4_act_ref(x)
    return q * (s * rs[:, None]).repeat_interleave(16, 1)


def quant_nvfp4_act(x: torch.Tensor):
    """(xq [M, K/2] packed e2m1, scale atoms, rs [M]) on the CUDA kernel."""
    M, K = x.shape
    xq = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    sf = torch.empty((M + 127) // 128 * (K // 64) * 512, dtype=torch.uint8, device=x.device)
    rs = torch.empty(max(M, 1), dtype=torch.float32, device=x.device)
    torch.ops._b200_C.quant_nvfp4_act(x, xq, sf, rs)
    launch_count.add(1)
    return xq, sf, rs


# ------------------------------------------------------------------ linears
class _WQLinear(Linear):
    fmt: str

    def _native(self, x) -> bool:
        if not x.is_cuda:
            return False
        _ext.require()
        return True

    def forward(self, x, out=None):
        M = x.shape[0]
        if out is None:
            out = torch.empty(M, self.out_features, device=x.device, dtype=torch.bfloat16)
        if not self._native(x):
            out.copy_((x.float() @ self.reference_weight().t()).to(out.dtype))
            return out
        if M <= WQ_MAX_M:
            torch.ops._b200_C.gemm_wq_out(out, x, self.raw, FMT_ID[self.fmt], self.scales,
                                          self.out_scale, 0, 0)
            launch_count.add(1)
        else:
            _lin.gemm(x, self.dequant(), out=out)
            launch_count.add(1)
        return out

    def dequant(self, with_global: bool = True) -> torch.Tensor:
        """bf16 weight from the native dequantiser (NVFP4: times the global
        scale unless ``with_global`` is False)."""
        w = torch.empty(self.out_features, self.in_features, device=self.raw.device,
                        dtype=torch.bfloat16)
        torch.ops._b200_C.dequant_weight(w, self.raw, FMT_ID[self.fmt], self.scales)
        launch_count.add(1)
        if with_global and self.out_scale != 1.0:
            w.mul_(self.out_scale)
        return w

    def reference_weight(self) -> torch.Tensor:
        """The dense weight this layer represents (fp32), for oracles."""
        return self.dequant_ref().float() * self.out_scale

    def reference_forward(self, x: torch.Tensor) -> torch.Tensor:
        """fp32 oracle of ``forward`` (weight-only formats: x times the dense weight)."""
        return x.float() @ self.reference_weight().t()

    def weight_bytes(self):
        return self.raw.numel() + self.scales.numel() * self.scales.element_size()


class Fp8BlockLinear(_WQLinear):
    fmt = "fp8"

    def __init__(self, w_fp8: torch.Tensor, scale_inv: torch.Tensor):
        self.out_features, self.in_features = w_fp8.shape
        self.raw = w_fp8.contiguous().view(torch.uint8)
        self.scales = scale_inv.float().contiguous()
        self.out_scale = 1.0

    def dequant_ref(self) -> torch.Tensor:
        q = self.raw.view(torch.float8_e4m3fn).float()
        s = self.scales.repeat_interleave(128, 0).repeat_interleave(128, 1)
        s = s[: self.out_features, : self.in_features]
        return (q * s).to(torch.bfloat16)

    def forward(self, x, out=None):
        if w8a8_enabled():
            if x.is_cuda and envs.get("VLLM_B200_FP8_GEMM"):
                _ext.require()
                return gemm_fp8(x, self.raw, self.scales, out)
            if not x.is_cuda:
                r = self.reference_forward(x).to(torch.bfloat16)
                if out is None:
                    return r
                out.copy_(r)
                return out
        return super().forward(x, out)

    def exact_weight(self) -> torch.Tensor:
        """fp32 dequantised weight without the bf16 rounding of ``dequant_ref``
        (what the W8A8 tensor-core path multiplies with)."""
        q = self.raw.view(torch.float8_e4m3fn).float()
        s = self.scales.repeat_interleave(128, 0).repeat_interleave(128, 1)
        return q * s[: self.out_features, : self.in_features]

    def reference_forward(self, x: torch.Tensor) -> torch.Tensor:
        if w8a8_enabled():
            return fp8_act_dequant_ref(x) @ self.exact_weight().t()
        return super().reference_forward(x)


class AwqLinear(_WQLinear):
    fmt = "awq"

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                 group: int = 128):
        assert group == 128, "the AWQ kernels serve group size 128"
        K = qweight.shape[0]
        N = qweight.shape[1] * 8
        self.out_features, self.in_features = N, K
        q = unpack_awq(qweight).t().contiguous()             # [N, K]
        z = unpack_awq(qzeros).t().float()                    # [N, K/128]
        s = scales.t().float()                                # [N, K/128]
        self.raw = (q[:, 0::2] | (q[:, 1::2] << 4)).to(torch.uint8).contiguous()
        s_bf = s.to(torch.bfloat16)
        zs_bf = (-z * s_bf.float()).to(torch.bfloat16)
        self.scales = torch.stack([s_bf, zs_bf], -1).view(N, -1).contiguous()
        self.out_scale = 1.0

    def dequant_ref(self) -> torch.Tensor:
        N, K = self.out_features, self.in_features
        lo = (self.raw & 0xF).to(torch.float64)
        hi = (self.raw >> 4).to(torch.float64)
        q = torch.stack([lo, hi], -1).view(N, K)
        sz = self.scales.view(N, K // 128, 2).double()
        s = sz[..., 0].repeat_interleave(128, 1)
        zs = sz[..., 1].repeat_interleave(128, 1)
        return (q * s + zs).float().to(torch.bfloat16)  # fp32 FMA == exact-in-fp64 then round


class Nvfp4Linear(_WQLinear):
    fmt = "nvfp4"

    def __init__(self, packed: torch.Tensor, block_scale: torch.Tensor, global_scale: float):
        self.out_features = packed.shape[0]
        self.in_features = packed.shape[1] * 2
        self.raw = packed.contiguous().view(torch.uint8)
        self.scales = block_scale.contiguous().view(torch.uint8)
        self.out_scale = float(global_scale)

    def dequant_ref(self, with_global: bool = False) -> torch.Tensor:
        N, K = self.out_features, self.in_features
        lut = E2M1.to(self.raw.device)
        q = torch.stack([lut[(self.raw & 0xF).long()], lut[(self.raw >> 4).long()]], -1).view(N, K)
        sc = self.scales.view(torch.float8_e4m3fn).float().repeat_interleave(16, 1)
        w = (q * sc).to(torch.bfloat16)
        if with_global:
            w = (w.float() * self.out_scale).to(torch.bfloat16)
        return w

    def exact_weight(self) -> torch.Tensor:
        """fp32 e2m1 x e4m3 block scale (no global scale, no bf16 rounding)."""
        N, K = self.out_features, self.in_features
        lut = E2M1.to(self.raw.device)
        q = torch.stack([lut[(self.raw & 0xF).long()], lut[(self.raw >> 4).long()]], -1).view(N, K)
        return q * self.scales.view(torch.float8_e4m3fn).float().repeat_interleave(16, 1)

    def sf_atoms(self) -> torch.Tensor:
        if getattr(self, "_atoms", None) is None or self._atoms.device != self.raw.device:
            self._atoms = nvfp4_sf_atoms(self.scales)
        return self._atoms

    def _w4a4(self, x) -> bool:
        return (w4a4_enabled() and self.in_features % 256 == 0 and
                self.out_features % 8 == 0)

    def forward(self, x, out=None):
        if self._w4a4(x):
            if x.is_cuda and envs.get("VLLM_B200_NVFP4_GEMM"):
                _ext.require()
                if out is None:
                    out = torch.empty(x.shape[0], self.out_features, dtype=torch.bfloat16,
                                      device=x.device)
                xq, sf, rs = quant_nvfp4_act(x)
                torch.ops._b200_C.gemm_nvfp4_out(out, xq, sf, rs, self.raw, self.sf_atoms(),
                                                 self.out_scale, -1)
                launch_count.add(1)
                return out
            if not x.is_cuda:
                r = self.reference_forward(x).to(torch.bfloat16)
                if out is None:
                    return r
                out.copy_(r)
                return out
        return super().forward(x, out)

    def reference_forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._w4a4(x):
            return (nvfp4_act_dequant_ref(x) @ self.exact_weight().t()) * self.out_scale
        return super().reference_forward(x)


def merge_nvfp4_parts(ws, ss, gs):
    """Row-concatenate NVFP4 parts (``weight`` uint8 ``[n_i, K/2]``, block
    scales e4m3 ``[n_i, K/16]``, global scale ``g_i``) under ONE global scale,
    the largest: each part's block scales are multiplied by ``g_i / g`` and
    rounded to e4m3 -- exact when the globals agree (ModelOpt exports fused
    projections and MoE experts that way), a rounding of the block scales
    otherwise."""
    g = max(gs)
    out = []
    for s, gi in zip(ss, gs):
        s = s.view(torch.float8_e4m3fn)
        if gi != g:
            s = (s.float() * (gi / g)).to(torch.float8_e4m3fn)
        out.append(s)
    return torch.cat(list(ws)), torch.cat(out), float(g)


def make_linear(fmt: str, w: torch.Tensor) -> _WQLinear:
    """Quantise a dense weight ``[N, K]`` into the given format (tests and
    random-init models)."""
    if fmt == "fp8":
        return Fp8BlockLinear(*quantize_fp8_block(w))
    if fmt == "awq":
        return AwqLinear(*quantize_awq(w))
    if fmt == "nvfp4":
        return Nvfp4Linear(*quantize_nvfp4(w))
    raise ValueError(fmt)


def enabled(fmt: str) -> bool:
    return {"fp8": envs.get("VLLM_B200_FP8_GEMM"), "awq": envs.get("VLLM_B200_AWQ_GEMM"),
            "nvfp4": envs.get("VLLM_B200_NVFP4_GEMM")}[fmt]
