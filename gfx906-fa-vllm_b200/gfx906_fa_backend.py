# SPDX-License-Identifier: Apache-2.0
"""vLLM v1 attention backend on the sm_100a paged-Q8 kernels.

Same plugin surface as the reference (extension/gfx906_fa_backend.py of
nick413-bit/gfx906-fa-vllm): registered as AttentionBackendEnum.CUSTOM by
`register()` (entry point `vllm.general_plugins: gfx906_fa =
gfx906_fa_backend:register`), the same class names, and the same KV-cache
shape as TritonAttentionBackend, (num_blocks, 2, block_size, num_kv_heads,
head_size), so the vLLM allocator is untouched.

Differences in how the cache is used:
  * The Q8_0 K rows live INSIDE the K half of each page of that allocation,
    densely packed as [block_size][Hkv][D/32*34] bytes at its start (136 of
    every 256 bytes at D = 128), written by one fused store kernel together
    with V.  There is no separate side buffer, so nothing can fall out of
    sync with it (the reference's side buffer did:
    tests/test_backend_vs_legacy.py).  Consequence: vLLM code that copies K
    pages as opaque bytes keeps working, code that reads K as 16-bit values
    does not.
  * V stays in the model dtype in the V half (GFX906_FA_V_FMT=fp16, default,
    the reference's numerics) or (GFX906_FA_V_FMT=q8_0) is stored as Q8_0
    page-transposed records right after the page's Q8_0 K rows, inside the
    K half, so a page's K and V are one contiguous byte range
    (gfx906_fa_paged.kv_cache_views).
  * forward writes straight into vLLM's output buffer in the model dtype:
    no fp32 upcast of the query, no padding, no per-sequence host loop.
  * GFX906_FA_LEGACY=1 keeps the reference's legacy design: 16-bit K/V in
    the cache (vLLM's own reshape_and_cache_flash) and K quantised on the
    fly in every forward.
"""
from __future__ import annotations

import os as _os
from dataclasses import dataclass, field
from typing import ClassVar

import torch

from vllm.config import VllmConfig
from vllm.config.cache import CacheDType
from vllm.logger import init_logger
from vllm.platforms.interface import DeviceCapability
from vllm.v1.attention.backend import (
    AttentionBackend,
    AttentionCGSupport,
    AttentionImpl,
    AttentionLayer,
    AttentionMetadataBuilder,
    AttentionType,
    CommonAttentionMetadata,
    MultipleOf,
)
from vllm.v1.kv_cache_interface import AttentionSpec

import gfx906_fa
from gfx906_fa_paged import forward_paged  # noqa: E402

logger = init_logger(__name__)

_V_FMT = _os.environ.get("GFX906_FA_V_FMT", "fp16").lower()


from gfx906_fa_paged import kv_cache_views, q8_row_bytes  # noqa: E402,F401  (cache layout)


# -----------------------------------------------------------------------------
# Metadata
# -----------------------------------------------------------------------------
@dataclass
class Gfx906FAMetadata:
    num_actual_tokens: int
    max_query_len: int
    max_seq_len: int
    query_start_loc: torch.Tensor      # [B+1] int32
    seq_lens: torch.Tensor             # [B]   int32
    block_table: torch.Tensor          # [B, max_num_blocks] int32
    slot_mapping: torch.Tensor         # [num_tokens] int64
    use_cascade: bool = False
    common_prefix_len: int = 0
    # host copies made once per step by the builder (shared by every layer):
    # exact query lengths and upper bounds of the context lengths
    query_lens_host: list | None = field(default=None)
    seq_lens_host: list | None = field(default=None)


class Gfx906FAMetadataBuilder(AttentionMetadataBuilder[Gfx906FAMetadata]):
    # Pure decode batches (one query token per sequence) can be captured in a
    # CUDA graph: the decode path reads lengths, positions and the block
    # table from device memory at run time and needs no host value that
    # changes between replays.  Mixed batches take host-sized prefill
    # staging and run eagerly.
    _cudagraph_support: ClassVar[AttentionCGSupport] = AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE

    def __init__(self, kv_cache_spec: AttentionSpec, layer_names: list[str], vllm_config: VllmConfig,
                 device: torch.device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        self.block_size = kv_cache_spec.block_size

    def build_for_cudagraph_capture(self, common_attn_metadata: CommonAttentionMetadata) -> Gfx906FAMetadata:
        # The kernels clamp each context to max_seq_len; a captured graph is
        # replayed with longer contexts later, so the bound it bakes in is the
        # block table's capacity.
        m = self.build(0, common_attn_metadata)
        m.max_seq_len = int(m.block_table.shape[1]) * self.block_size
        return m

    def build(self, common_prefix_len: int, common_attn_metadata: CommonAttentionMetadata,
              fast_build: bool = False) -> Gfx906FAMetadata:
        m = common_attn_metadata
        qlens = slens = None
        qsl_cpu = getattr(m, "query_start_loc_cpu", None)
        if qsl_cpu is not None:
            q = qsl_cpu.tolist()
            qlens = [q[i + 1] - q[i] for i in range(len(q) - 1)]
        ub = getattr(m, "seq_lens_cpu_upper_bound", None)
        if ub is not None:
            slens = ub.tolist()
        return Gfx906FAMetadata(
            num_actual_tokens=m.num_actual_tokens,
            max_query_len=m.max_query_len,
            max_seq_len=m.max_seq_len,
            query_start_loc=m.query_start_loc,
            seq_lens=m.seq_lens,
            block_table=m.block_table_tensor,
            slot_mapping=m.slot_mapping,
            use_cascade=(common_prefix_len > 0),
            common_prefix_len=common_prefix_len,
            query_lens_host=qlens,
            seq_lens_host=slens,
        )


# -----------------------------------------------------------------------------
# Backend
# -----------------------------------------------------------------------------
class Gfx906FABackend(AttentionBackend):
    accept_output_buffer: bool = True
    supported_dtypes: ClassVar[list[torch.dtype]] = [torch.float16, torch.bfloat16]
    supported_kv_cache_dtypes: ClassVar[list[CacheDType]] = ["auto", "float16", "half", "bfloat16"]
    forward_includes_kv_cache_update: bool = False

    @staticmethod
    def get_supported_kernel_block_sizes() -> list[int | MultipleOf]:
        return [MultipleOf(16)]

    @classmethod
    def supports_block_size(cls, block_size: int | None) -> bool:
        if block_size is None:
            return True
        return block_size % 16 == 0

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls() -> type["Gfx906FAImpl"]:
        return Gfx906FAImpl

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        if block_size % 16 != 0:
            raise ValueError("Block size must be a multiple of 16.")
        return (num_blocks, 2, block_size, num_kv_heads, head_size)

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension: bool = False) -> tuple[int, ...]:
        if include_num_layers_dimension:
            return (1, 0, 2, 3, 4, 5)
        return (0, 1, 2, 3, 4)

    @staticmethod
    def use_cascade_attention(*args, **kwargs) -> bool:
        return False

    @staticmethod
    def get_builder_cls() -> type["Gfx906FAMetadataBuilder"]:
        return Gfx906FAMetadataBuilder

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size == 128

    @classmethod
    def supports_mm_prefix(cls) -> bool:
        return False

    @classmethod
    def supports_sink(cls) -> bool:
        return True

    @classmethod
    def supports_attn_type(cls, attn_type: str) -> bool:
        return attn_type == AttentionType.DECODER

    @classmethod
    def supports_alibi_sqrt(cls) -> bool:
        return False

    @classmethod
    def supports_compute_capability(cls, capability: DeviceCapability) -> bool:
        return capability.major == 10


# -----------------------------------------------------------------------------
# Impl
# -----------------------------------------------------------------------------
class Gfx906FAImpl(AttentionImpl):

    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int,
                 alibi_slopes: list[float] | None, sliding_window: int | None, kv_cache_dtype: str,
                 logits_soft_cap: float | None = None, attn_type: AttentionType = AttentionType.DECODER,
                 kv_sharing_target_layer_name: int | None = None, sinks: torch.Tensor | None = None,
                 use_alibi_sqrt: bool = False) -> None:
        if alibi_slopes is not None:
            raise NotImplementedError("GFX906_FA: alibi_slopes is not supported")
        # Sliding window, logit soft-cap and sinks are computed by the kernels
        # (the reference rejected all three).  vLLM passes the window as its
        # size: a query at position p sees keys p - sliding_window + 1 .. p.
        if sliding_window is not None and sliding_window <= 0:
            raise ValueError(f"GFX906_FA: sliding_window must be positive, got {sliding_window}")
        if sinks is not None and tuple(sinks.shape) != (num_heads,):
            raise ValueError(f"GFX906_FA: sinks must have shape ({num_heads},), got {tuple(sinks.shape)}")
        if attn_type != AttentionType.DECODER:
            raise NotImplementedError(f"GFX906_FA: attn_type={attn_type} is not supported")
        if head_size != 128:
            raise NotImplementedError("GFX906_FA: head_size must be 128")
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = float(scale)
        self.num_kv_heads = num_kv_heads
        self.kv_cache_dtype = kv_cache_dtype
        self.attn_type = attn_type
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        self.num_queries_per_kv = num_heads // num_kv_heads
        self.sliding_window = int(sliding_window) if sliding_window else 0
        self.logits_soft_cap = float(logits_soft_cap) if logits_soft_cap else 0.0
        self.sinks = sinks
        self._legacy = _os.environ.get("GFX906_FA_LEGACY", "0") == "1"
        self._v_fmt = "q8_0" if _V_FMT in ("q8", "q8_0") else "fp16"

    def fused_output_quant_supported(self, quant_key):
        # static per-tensor fp8 (e4m3) output quantisation, fused into the
        # attention epilogues (not on the legacy path)
        from vllm.model_executor.layers.quantization.utils.quant_utils import kFp8StaticTensorSym
        return not self._legacy and quant_key == kFp8StaticTensorSym

    def fused_rope_kvcache_supported(self):
        # RoPE is fused into the Q8_0 store kernel (the legacy mode keeps
        # vLLM's own cache layout and ops)
        return not self._legacy

    def do_rope_and_kv_cache_update(self, layer: AttentionLayer, query: torch.Tensor, key: torch.Tensor,
                                    value: torch.Tensor, positions: torch.Tensor, cos_sin_cache: torch.Tensor,
                                    is_neox: bool, kv_cache: torch.Tensor, layer_slot_mapping: torch.Tensor):
        """vLLM's RoPE + KV-cache fusion hook: query and key are rotated in
        place (fp32 arithmetic, one rounding to the model dtype) and the
        rotated key is quantised into the cache with V, in one kernel."""
        slots = layer_slot_mapping if layer_slot_mapping.dtype == torch.int64 else layer_slot_mapping.to(torch.int64)
        n = slots.shape[0]
        D = self.head_size
        q3 = query.view(query.shape[0], -1, D)
        k3 = key.view(key.shape[0], -1, D)
        v3 = value.view(value.shape[0], -1, D)
        pos = positions if positions.dtype == torch.int64 else positions.to(torch.int64)
        k_q8, v = kv_cache_views(kv_cache, self._v_fmt)
        gfx906_fa.rope_store_kv(q3[:n], k3[:n], v3[:n], pos, cos_sin_cache, bool(is_neox), slots, k_q8, v,
                                3 if self._v_fmt == "q8_0" else 1)

    # ------------------------------------------------------------------
    # KV cache write
    # ------------------------------------------------------------------
    def do_kv_cache_update(self, layer: AttentionLayer, key: torch.Tensor, value: torch.Tensor,
                           kv_cache: torch.Tensor, slot_mapping: torch.Tensor):
        slots = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
        if self._legacy:
            import vllm._custom_ops  # noqa: F401  (registers torch.ops._C_cache_ops)
            key_cache, value_cache = kv_cache.unbind(1)
            torch.ops._C_cache_ops.reshape_and_cache_flash(
                key, value, key_cache, value_cache, slots, self.kv_cache_dtype, layer._k_scale, layer._v_scale)
            return
        n = slots.shape[0]
        k_q8, v = kv_cache_views(kv_cache, self._v_fmt)
        gfx906_fa.store_kv(key[:n], value[:n], slots, k_q8, v, 3 if self._v_fmt == "q8_0" else 1)

    # ------------------------------------------------------------------
    # Forward
    # ------------------------------------------------------------------
    def forward(self, layer: torch.nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                kv_cache: torch.Tensor, attn_metadata: Gfx906FAMetadata, output: torch.Tensor | None = None,
                output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        assert output is not None, "Output tensor must be provided."
        if output_block_scale is not None:
            raise NotImplementedError("GFX906_FA: block-scaled output quantization is not supported")
        if output_scale is not None and self._legacy:
            raise NotImplementedError("GFX906_FA: output quantization needs the Q8_0 cache path (GFX906_FA_LEGACY=0)")
        if attn_metadata is None:
            return output.fill_(0)                 # profiling run
        assert not attn_metadata.use_cascade, "GFX906_FA: cascade attention is not supported"
        n = attn_metadata.num_actual_tokens
        q = query[:n]
        out = output[:n].view(n, self.num_heads, self.head_size)
        if self._legacy:
            key_cache, value_cache = kv_cache.unbind(1)
            res = forward_paged(q, key_cache, value_cache, attn_metadata.block_table, attn_metadata.seq_lens,
                                attn_metadata.query_start_loc, attn_metadata.max_query_len,
                                attn_metadata.max_seq_len, scale=self.scale, key_cache_q8=None,
                                softcap=self.logits_soft_cap, sliding_window=self.sliding_window,
                                sinks=self._sinks_f32())
            out.copy_(res.view(n, self.num_heads, self.head_size))
            return output
        k_q8, v = kv_cache_views(kv_cache, self._v_fmt)
        forward_paged(q, None, v, attn_metadata.block_table, attn_metadata.seq_lens,
                      attn_metadata.query_start_loc, attn_metadata.max_query_len, attn_metadata.max_seq_len,
                      scale=self.scale, key_cache_q8=k_q8, out=out,
                      query_lens_host=attn_metadata.query_lens_host, seq_lens_host=attn_metadata.seq_lens_host,
                      softcap=self.logits_soft_cap, sliding_window=self.sliding_window, sinks=self._sinks_f32(),
                      output_scale=output_scale)
        return output

    def _sinks_f32(self):
        """The sinks as fp32 on the layer's device, converted once."""
        if self.sinks is None:
            return None
        if self.sinks.dtype != torch.float32 or not self.sinks.is_contiguous():
            self.sinks = self.sinks.to(torch.float32).contiguous()
        return self.sinks


# -----------------------------------------------------------------------------
# Registration as AttentionBackendEnum.CUSTOM
# -----------------------------------------------------------------------------
def register() -> None:
    """Register Gfx906FABackend as AttentionBackendEnum.CUSTOM (reference:
    extension/gfx906_fa_backend.py:536-549).  Called by vLLM's general-plugin
    loader in every process, and once more on import."""
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    register_backend(AttentionBackendEnum.CUSTOM, f"{__name__}.Gfx906FABackend")
    logger.info("GFX906_FA backend registered as AttentionBackendEnum.CUSTOM")


register()
