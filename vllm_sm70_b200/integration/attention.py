"""vLLM attention backend over the B200 paged attention kernels.

Registered into the ``AttentionBackendEnum.CUSTOM`` slot. KV cache shape is
``(num_blocks, 2, num_kv_heads, block_size, head_size)``: K and V of one
block sit next to each other and each (block, head) is a dense
``block_size x head_size`` tile, which the kernels read with a block stride.
Decode-only batches use the decode kernel (GQA-packed rows, warps split the
keys, split-KV across CTAs for small batches); any batch with a multi-token
query uses the prefill kernel, which handles chunked prefill and mixed batches.

Reference parity: ``FlashAttnV100Backend`` / ``MetadataBuilder`` / ``Impl``
(``sm70/vllm_sm70/attention/flash_v100/backend.py:39-143``,
``metadata.py:66-296``, ``impl.py:59-186``), registered the same way
(``sm70/vllm_sm70/attention/__init__.py:26-37``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import ClassVar

import torch

from .. import _ext
from ..ops import attention as A

BACKEND_NAME = "B200_PAGED"
SUPPORTED_HEAD_SIZES = (64, 128, 256)


def _vllm():
    from vllm.v1.attention import backend as vb

    return vb


@dataclass
class B200AttentionMetadata:
    num_actual_tokens: int
    max_query_len: int
    max_seq_len: int
    query_start_loc: torch.Tensor
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    decode_only: bool
    num_splits: int = 1
    part_o: torch.Tensor | None = None
    part_ml: torch.Tensor | None = None


def _make_classes():
    vb = _vllm()

    class B200AttentionMetadataBuilder(vb.AttentionMetadataBuilder):
        _cudagraph_support: ClassVar = vb.AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE

        def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
            super().__init__(kv_cache_spec, layer_names, vllm_config, device)
            mc = vllm_config.model_config
            self.num_heads_q = mc.get_num_attention_heads(vllm_config.parallel_config)
            self.num_heads_kv = mc.get_num_kv_heads(vllm_config.parallel_config)
            self.head_dim = mc.get_head_size()
            props = torch.cuda.get_device_properties(device) if torch.cuda.is_available() else None
            self.num_sms = props.multi_processor_count if props else 148
            self.max_splits = 16
            mx = max(1, vllm_config.scheduler_config.max_num_seqs)
            self.part_o = torch.empty(self.max_splits, mx, self.num_heads_q, self.head_dim,
                                      dtype=torch.float32, device=device)
            self.part_ml = torch.empty(self.max_splits, mx, self.num_heads_q, 2,
                                       dtype=torch.float32, device=device)

        def _splits(self, num_reqs: int) -> int:
            work = max(1, num_reqs * self.num_heads_kv)
            return max(1, min(self.max_splits, math.ceil(2 * self.num_sms / work)))

        def build(self, common_prefix_len, common_attn_metadata, fast_build=False):
            cam = common_attn_metadata
            decode_only = cam.max_query_len == 1
            ns = self._splits(cam.num_reqs) if decode_only else 1
            if decode_only and cam.num_actual_tokens > self.part_o.shape[1]:
                ns = 1
            return B200AttentionMetadata(
                num_actual_tokens=cam.num_actual_tokens, max_query_len=cam.max_query_len,
                max_seq_len=cam.max_seq_len, query_start_loc=cam.query_start_loc,
                seq_lens=cam.seq_lens, block_table=cam.block_table_tensor,
                slot_mapping=cam.slot_mapping, decode_only=decode_only, num_splits=ns,
                part_o=self.part_o if ns > 1 else None, part_ml=self.part_ml if ns > 1 else None)

        def build_for_cudagraph_capture(self, common_attn_metadata):
            md = self.build(0, common_attn_metadata)
            md.seq_lens.fill_(1)
            return md

    class B200AttentionImpl(vb.AttentionImpl):
        def __init__(self, num_heads, head_size, scale, num_kv_heads, alibi_slopes,
                     sliding_window, kv_cache_dtype, logits_soft_cap=None,
                     attn_type=vb.AttentionType.DECODER, kv_sharing_target_layer_name=None,
                     sinks=None, **kw):
            if alibi_slopes is not None:
                raise NotImplementedError("B200 attention: ALiBi is not supported")
            if logits_soft_cap:
                raise NotImplementedError("B200 attention: logit soft-capping is not supported")
            if kv_cache_dtype not in ("auto", "bfloat16"):
                raise NotImplementedError("B200 attention: bf16 KV cache only")
            if attn_type != vb.AttentionType.DECODER:
                raise NotImplementedError("B200 attention: decoder self-attention only")
            self.num_heads = num_heads
            self.head_size = head_size
            self.scale = float(scale)
            self.num_kv_heads = num_kv_heads
            self.window = int(sliding_window) if sliding_window else 0
            self.sinks = sinks
            self.kv_sharing_target_layer_name = kv_sharing_target_layer_name

        def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
            if self.kv_sharing_target_layer_name is not None:
                return
            kc, vc = kv_cache.unbind(1)
            kv_cache_write(key, value, kc, vc, slot_mapping)

        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                    output_scale=None, output_block_scale=None):
            if output_scale is not None or output_block_scale is not None:
                raise NotImplementedError("B200 attention: fused output quant unsupported")
            if attn_metadata is None:
                return output.fill_(0)
            md = attn_metadata
            n = md.num_actual_tokens
            kc, vc = kv_cache.unbind(1)
            q = query[:n].view(n, self.num_heads, self.head_size)
            out = output[:n].view(n, self.num_heads, self.head_size)
            sinks = self.sinks.float() if self.sinks is not None else None
            A.paged_attention(out, q, kc, vc, md.block_table, md.seq_lens, md.query_start_loc,
                              md.max_query_len, self.scale, self.window, sinks, md.decode_only,
                              md.num_splits, md.part_o, md.part_ml)
            return output

    class B200AttentionBackend(vb.AttentionBackend):
        accept_output_buffer: bool = True
        forward_includes_kv_cache_update: bool = False
        supported_dtypes: ClassVar = [torch.bfloat16]
        supported_kv_cache_dtypes: ClassVar = ["auto", "bfloat16"]

        @staticmethod
        def get_name() -> str:
            return "CUSTOM"

        @staticmethod
        def get_impl_cls():
            return B200AttentionImpl

        @staticmethod
        def get_builder_cls():
            return B200AttentionMetadataBuilder

        @staticmethod
        def get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size,
                               cache_dtype_str="auto"):
            if block_size < 8 or block_size & (block_size - 1):
                raise ValueError("B200 attention: block size must be a power of two >= 8")
            return (num_blocks, 2, num_kv_heads, block_size, head_size)

        @staticmethod
        def get_supported_kernel_block_sizes():
            return [16, 32, 64, 128]

        @classmethod
        def supports_head_size(cls, head_size: int) -> bool:
            return head_size in SUPPORTED_HEAD_SIZES

        @classmethod
        def supports_sink(cls) -> bool:
            return True

        @classmethod
        def supports_compute_capability(cls, capability) -> bool:
            return tuple(capability) >= (10, 0) and tuple(capability) < (11, 0)

        @staticmethod
        def use_cascade_attention(*args, **kwargs) -> bool:
            return False

    return B200AttentionMetadataBuilder, B200AttentionImpl, B200AttentionBackend


_classes = None


def __getattr__(name):
    global _classes
    if name in ("B200AttentionMetadataBuilder", "B200AttentionImpl", "B200AttentionBackend"):
        if _classes is None:
            _classes = _make_classes()
        return dict(zip(("B200AttentionMetadataBuilder", "B200AttentionImpl",
                         "B200AttentionBackend"), _classes))[name]
    raise AttributeError(name)


def kv_cache_write(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Write ``key/value [T, Hkv, D]`` into paged caches at ``slot_mapping``."""
    if key.is_cuda:
        _ext.require()
        torch.ops._b200_C.kv_cache_write(key, value, k_cache, v_cache, slot_mapping.long())
        return
    bs = k_cache.shape[2]
    for t in range(key.shape[0]):
        s = int(slot_mapping[t])
        if s < 0:
            continue
        k_cache[s // bs, :, s % bs] = key[t]
        v_cache[s // bs, :, s % bs] = value[t]


def select(head_size: int, dtype: torch.dtype, has_sinks: bool = False) -> bool:
    """Backend admission (reference: ``attention/__init__.py:40-102``)."""
    return head_size in SUPPORTED_HEAD_SIZES and dtype == torch.bfloat16


def register() -> None:
    """Plugin area hook: register into vLLM's CUSTOM attention slot."""
    try:
        from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    except Exception:  # noqa: BLE001 - vLLM not importable: nothing to register
        return
    register_backend(AttentionBackendEnum.CUSTOM,
                     "vllm_sm70_b200.integration.attention.B200AttentionBackend")
