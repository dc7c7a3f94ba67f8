"""Attention backend ABI mirror and the B200 backend behind it.

Mirrors ``layers/attention/backends/attention_backend.py`` (enum ``:13-17``,
capability/support/selection dataclasses ``:20-40``, the unavailable error
``:43-58``, ``validate_bshd_qkv`` ``:61-91``, ``AttentionBackend`` ``:94-120``,
``AttentionMetadata`` ``:123-136``, ``AttentionImpl`` ``:150-182``) so that the
reference's callers (``models/dits/eraserdit_attention.py:287-289``,
``layers/attention/sequence_parallel.py:242-247``,
``models/adapters/eraserdit/nccl_sequence.py:259-260``) can hold a
:class:`B200AttentionImpl` where they held ``SDPAImpl``
(``layers/attention/backends/sdpa.py:56-80``).

The B200 backend is selected explicitly; ``probe`` reports unsupported
capabilities instead of falling back, and ``forward`` raises on anything the
native kernel does not implement.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from enum import Enum
from typing import Any

import torch

from . import _native


class AttentionBackendEnum(str, Enum):
    TORCH_SDPA = "torch_sdpa"
    FLASH_ATTN = "flash_attn"
    SAGE_ATTN = "sage_attn"
    SAGE_FP8 = "sage_fp8"
    B200_NATIVE = "b200_native"
    B200_FP8 = "b200_fp8"


@dataclass(frozen=True)
class AttentionCapability:
    device: torch.device
    dtype: torch.dtype
    head_size: int
    causal: bool = False
    has_attn_mask: bool = False


@dataclass(frozen=True)
class AttentionSupport:
    supported: bool
    reason: str | None = None


class AttentionBackendUnavailableError(RuntimeError):
    def __init__(self, requested, reason: str) -> None:
        name = requested.value if isinstance(requested, AttentionBackendEnum) else requested
        self.requested = name
        self.reason = reason
        super().__init__(f"Attention backend {name!r} is unavailable: {reason}")


def validate_bshd_qkv(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> None:
    """Same checks and messages as the reference's ``validate_bshd_qkv``."""
    for name, tensor in (("query", query), ("key", key), ("value", value)):
        if tensor.ndim != 4:
            raise ValueError(f"{name} must use BSHD rank-4 layout, got rank {tensor.ndim}")
    if query.shape[0] != key.shape[0] or query.shape[0] != value.shape[0]:
        raise ValueError("Q/K/V batch dimensions must match")
    if query.shape[3] != key.shape[3] or query.shape[3] != value.shape[3]:
        raise ValueError("Q/K/V head_dim dimensions must match")
    if query.dtype != key.dtype or query.dtype != value.dtype:
        raise ValueError("Q/K/V dtype values must match")
    if query.device != key.device or query.device != value.device:
        raise ValueError("Q/K/V device values must match")
    if key.shape[1] != value.shape[1]:
        raise ValueError("K/V sequence dimensions must match")
    if key.shape[2] != value.shape[2]:
        raise ValueError("K/V heads must match")
    if query.shape[2] <= 0 or key.shape[2] <= 0 or query.shape[2] % key.shape[2] != 0:
        raise ValueError("Q heads must equal K/V heads or be a positive integer multiple")


@dataclass
class AttentionMetadata:
    current_timestep: int = 0
    attn_mask: torch.Tensor | None = None

    def asdict_zerocopy(self, skip_fields: set[str] | None = None) -> dict[str, Any]:
        skip = skip_fields or set()
        out: dict[str, Any] = {}
        if "current_timestep" not in skip:
            out["current_timestep"] = self.current_timestep
        if "attn_mask" not in skip:
            out["attn_mask"] = self.attn_mask
        return out


class AttentionBackend(ABC):
    accept_output_buffer: bool = False

    @staticmethod
    @abstractmethod
    def probe(capability: AttentionCapability) -> AttentionSupport: ...

    @staticmethod
    @abstractmethod
    def get_enum() -> AttentionBackendEnum: ...

    @staticmethod
    @abstractmethod
    def get_impl_cls() -> type["AttentionImpl"]: ...

    @staticmethod
    def get_metadata_cls() -> type[AttentionMetadata]:
        return AttentionMetadata

    @staticmethod
    def get_builder_cls():
        return None


class AttentionImpl(ABC):
    @abstractmethod
    def __init__(self, num_heads: int, head_size: int, softmax_scale: float, causal: bool = False,
                 num_kv_heads: int | None = None, prefix: str = "", **extra_impl_args) -> None: ...

    def preprocess_qkv(self, qkv: torch.Tensor, attn_metadata) -> torch.Tensor:
        return qkv

    def postprocess_output(self, output: torch.Tensor, attn_metadata) -> torch.Tensor:
        return output

    @abstractmethod
    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                attn_metadata) -> torch.Tensor: ...


def _is_sm100(device: torch.device) -> bool:
    if device.type != "cuda" or not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(device) == (10, 0)


class B200AttentionBackend(AttentionBackend):
    """tcgen05/TMEM attention for sm_100a, head_dim 64, BF16, non-causal, unmasked."""

    accept_output_buffer: bool = True

    @staticmethod
    def probe(capability: AttentionCapability) -> AttentionSupport:
        if capability.device.type != "cuda":
            return AttentionSupport(False, "b200_native requires a CUDA device")
        if not _is_sm100(capability.device):
            return AttentionSupport(False, "b200_native requires compute capability 10.0 (B200)")
        if capability.dtype != torch.bfloat16:
            return AttentionSupport(False, "b200_native requires bfloat16 Q/K/V")
        if capability.head_size != 64:
            return AttentionSupport(False, "b200_native supports head_size 64")
        if capability.causal:
            return AttentionSupport(False, "b200_native is non-causal")
        if capability.has_attn_mask:
            return AttentionSupport(False, "b200_native does not take an attention mask")
        try:
            _native.load()
        except (RuntimeError, OSError) as error:
            return AttentionSupport(False, str(error))
        return AttentionSupport(True)

    @staticmethod
    def get_supported_head_sizes() -> list[int]:
        return [64]

    @staticmethod
    def get_enum() -> AttentionBackendEnum:
        return AttentionBackendEnum.B200_NATIVE

    @staticmethod
    def get_impl_cls() -> type["B200AttentionImpl"]:
        return B200AttentionImpl


def _check_operand(name: str, t: torch.Tensor) -> None:
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have a contiguous head_dim")
    if t.data_ptr() % 16 or any(s % 8 for s in t.stride()[:-1]):
        raise ValueError(f"{name} needs 16-byte aligned rows (strides multiple of 8 elements)")


def _segmented_call(fn_name: str, query, key, value, out, softmax_scale, *, batch, heads,
                    seg_len, nseg, seg_lens, q_strides, k_strides, v_strides, o_strides,
                    extra=()) -> None:
    """Enqueue an attention entry point with segmented strides (token, head,
    batch, segment) for q / k / v / out."""
    lib = _native.load()
    device = query.device
    lens = None
    if seg_lens is not None:
        import ctypes
        lens = (ctypes.c_int32 * nseg)(*seg_lens)
    with torch.cuda.device(device):
        rc = getattr(lib, fn_name)(
            query.data_ptr(), key.data_ptr(), value.data_ptr(), *q_strides, *k_strides,
            *v_strides, batch, heads, seg_len, nseg, lens, 64, float(softmax_scale),
            out.data_ptr(), *o_strides, *extra,
            _native.status_word(device).data_ptr(), _native.stream_handle(device))
    _native.check(rc, fn_name)


def fp8_workspace(device: torch.device, batch: int, heads: int, seg_len: int, nseg: int) -> tuple:
    lib = _native.load()
    nbytes = int(lib.erd_attn_fp8_workspace_bytes(batch, heads, seg_len, nseg))
    return _native.workspace(device, nbytes), nbytes


def attention_bshd(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   softmax_scale: float, out: torch.Tensor | None = None,
                   precision: str = "bf16") -> torch.Tensor:
    """softmax(Q K^T * scale) V on BSHD tensors through ``erd_attn_fwd_bf16``
    (or ``erd_attn_fwd_fp8`` with ``precision="fp8"``)."""
    validate_bshd_qkv(query, key, value)
    if query.shape != key.shape:
        raise ValueError("b200_native self-attention needs equal Q and K/V shapes")
    if query.dtype != torch.bfloat16 or not query.is_cuda or query.shape[-1] != 64:
        raise ValueError("b200_native needs CUDA bfloat16 BSHD tensors with head_dim 64")
    if precision not in ("bf16", "fp8"):
        raise ValueError("precision must be bf16 or fp8")
    batch, seq, heads, dim = query.shape
    if out is None:
        out = torch.empty_like(query, memory_format=torch.contiguous_format)
    for name, t in (("query", query), ("key", key), ("value", value), ("out", out)):
        _check_operand(name, t)
    if seq == 0 or batch == 0:
        return out
    st = lambda t: (t.stride(1), t.stride(2), t.stride(0), 0)
    extra = ()
    if precision == "fp8":
        extra = fp8_workspace(query.device, batch, heads, seq, 1)
    _segmented_call("erd_attn_fwd_bf16" if precision == "bf16" else "erd_attn_fwd_fp8",
                    query, key, value, out, softmax_scale, batch=batch, heads=heads, seg_len=seq,
                    nseg=1, seg_lens=None, q_strides=st(query), k_strides=st(key),
                    v_strides=st(value), o_strides=st(out), extra=extra)
    return out


class B200AttentionImpl(AttentionImpl):
    def __init__(self, num_heads: int, head_size: int, softmax_scale: float, causal: bool = False,
                 num_kv_heads: int | None = None, prefix: str = "", **extra_impl_args) -> None:
        if causal:
            raise ValueError("b200_native attention is non-causal")
        self.num_heads = num_heads
        self.head_size = head_size
        self.causal = False
        self.softmax_scale = float(softmax_scale)
        self.dropout = float(extra_impl_args.get("dropout_p", 0.0))
        if self.dropout:
            raise ValueError("b200_native attention does not implement dropout")
        self.prefix = prefix
        self.calls = 0

    def forward(self, query, key, value, attn_metadata) -> torch.Tensor:
        if attn_metadata is not None and getattr(attn_metadata, "attn_mask", None) is not None:
            raise ValueError("b200_native attention does not take an attention mask")
        self.calls += 1
        return attention_bshd(query, key, value, self.softmax_scale)

    def report(self) -> dict:
        return {"backend": "b200_native", "calls": self.calls}


class B200FP8AttentionBackend(AttentionBackend):
    """SageAttention-style FP8 attention (E4M3 Q/K/P/V, FP32 accumulation) for sm_100a."""

    accept_output_buffer: bool = True

    @staticmethod
    def probe(capability: AttentionCapability) -> AttentionSupport:
        return B200AttentionBackend.probe(capability)

    @staticmethod
    def get_supported_head_sizes() -> list[int]:
        return [64]

    @staticmethod
    def get_enum() -> AttentionBackendEnum:
        return AttentionBackendEnum.B200_FP8

    @staticmethod
    def get_impl_cls() -> type["B200FP8AttentionImpl"]:
        return B200FP8AttentionImpl


class B200FP8AttentionImpl(B200AttentionImpl):
    """Drop-in for ``SageFP8AttentionImpl`` (``layers/attention/backends/sage_fp8.py:100-219``):
    same constructor arguments (``pv_accum_dtype`` must be FP32 accumulation;
    the quantization granularity is the per-128-token-block scheme)."""

    def __init__(self, num_heads: int, head_size: int, softmax_scale: float, causal: bool = False,
                 num_kv_heads: int | None = None, prefix: str = "",
                 pv_accum_dtype: str = "fp32+fp32", qk_quant_gran: str = "per_block",
                 **extra_impl_args) -> None:
        if pv_accum_dtype != "fp32+fp32":
            raise ValueError("b200_fp8 accumulates P V in FP32 only")
        if qk_quant_gran not in ("per_block", "per_thread", "per_warp"):
            raise ValueError("unsupported QK quantization granularity")
        super().__init__(num_heads, head_size, softmax_scale, causal, num_kv_heads, prefix,
                         **extra_impl_args)
        self.pv_accum_dtype = pv_accum_dtype
        self.qk_quant_gran = "per_block"

    def forward(self, query, key, value, attn_metadata) -> torch.Tensor:
        if attn_metadata is not None and getattr(attn_metadata, "attn_mask", None) is not None:
            raise ValueError("b200_fp8 attention does not take an attention mask")
        self.calls += 1
        return attention_bshd(query, key, value, self.softmax_scale, precision="fp8")

    def report(self) -> dict:
        return {"backend": "b200_fp8", "calls": self.calls, "qk_quant_granularity": "per_block",
                "pv_accum_dtype": self.pv_accum_dtype, "smooth_k": True}
