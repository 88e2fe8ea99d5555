"""B200 drop-in for the reference's ``MixedPrecisionTransformer``.

Same constructor arguments, module tree, parameter names and shapes as
mixed_precision/transformer.py:327-699, so ``copy_mixed_model_weights`` loads
into it with ``strict=True`` and ``mixed_precision_benchmark.py`` can use it
unchanged apart from the import.  ``forward`` makes one call into
libtt_b200.so (``tt_model_forward``), which launches the hand-written sm_100a
kernels for every op of every layer; there is no PyTorch, Triton or CPU
compute path behind it.
"""

from __future__ import annotations

import copy
import ctypes
import itertools
import weakref
from dataclasses import dataclass
from typing import Dict, Optional, Sequence

import torch
import torch.nn as nn

from . import _lib


@dataclass(frozen=True)
class TransformerConfig:
    """Field-for-field the reference's TransformerConfig (torch_transformer_benchmark.py:106-133)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        for name in ("batch_size", "seq_len", "d_model", "num_heads", "ffn_dim", "num_layers"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by num_heads ({self.num_heads})"
            )


class MixedPrecisionSelfAttention(nn.Module):
    """Parameter holder matching mixed_precision/transformer.py:35-66 (qkv_proj, out_proj)."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim**-0.5
        self.qkv_proj = nn.Linear(d_model, 3 * d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    def convert_projections_to_fp16(self) -> None:
        self.qkv_proj.half()
        self.out_proj.half()


class MixedPrecisionTransformerBlock(nn.Module):
    """Parameter holder matching mixed_precision/transformer.py:281-324."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = MixedPrecisionSelfAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def convert_projections_to_fp16(self) -> None:
        self.attention.convert_projections_to_fp16()
        self.ffn_in.half()
        self.ffn_out.half()


class _DevicePlan:
    """libtt_b200 model handle + workspace for one device and one set of weights."""

    def __init__(self, model: "B200Transformer", device: torch.device) -> None:
        cfg = model.config
        self.device = device
        self.key = model._weights_key()
        self._keep = []  # tensors whose pointers the C handle holds
        layers = (_lib.LayerWeights * cfg.num_layers)()
        for i, layer in enumerate(model.layers):
            att = layer.attention
            nxt = model.layers[i + 1].norm1 if i + 1 < cfg.num_layers else model.final_norm
            lw = layers[i]
            lw.w_qkv = self._w16(att.qkv_proj.weight)
            lw.b_qkv = self._b32(model, f"layers.{i}.attention.qkv_proj", att.qkv_proj.bias)
            lw.w_out = self._w16(att.out_proj.weight)
            lw.b_out = self._b32(model, f"layers.{i}.attention.out_proj", att.out_proj.bias)
            lw.ln_attn_w = self._f32(layer.norm2.weight)
            lw.ln_attn_b = self._f32(layer.norm2.bias)
            lw.w_ffn_in = self._w16(layer.ffn_in.weight)
            lw.b_ffn_in = self._b32(model, f"layers.{i}.ffn_in", layer.ffn_in.bias)
            lw.w_ffn_out = self._w16(layer.ffn_out.weight)
            lw.b_ffn_out = self._b32(model, f"layers.{i}.ffn_out", layer.ffn_out.bias)
            lw.ln_next_w = self._f32(nxt.weight)
            lw.ln_next_b = self._f32(nxt.bias)
        desc = _lib.ModelDesc()
        desc.d_model = cfg.d_model
        desc.heads = cfg.num_heads
        desc.ffn_dim = cfg.ffn_dim
        desc.num_layers = cfg.num_layers
        desc.causal = int(bool(cfg.causal))
        desc.eps = float(model.layers[0].norm1.eps)
        desc.ln0_w = self._f32(model.layers[0].norm1.weight)
        desc.ln0_b = self._f32(model.layers[0].norm1.bias)
        desc.layers = layers
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(_lib.lib().tt_model_create(ctypes.byref(desc), ctypes.byref(handle)))
        self.handle = handle
        self._ws_ptr = 0
        self._ws_bytes = 0

    def _hold(self, t: torch.Tensor) -> int:
        if t.device != self.device:
            raise ValueError(f"parameter on {t.device}, model running on {self.device}")
        self._keep.append(t)
        return t.data_ptr()

    def _w16(self, w: torch.Tensor) -> int:
        if w.dtype != torch.float16:
            raise RuntimeError(
                "projection weights must be FP16: call convert_projections_to_fp16() after moving "
                "the model to the GPU (mixed_precision_benchmark.py does this)"
            )
        return self._hold(w.detach().contiguous())

    def _f32(self, t: torch.Tensor) -> int:
        if t.dtype != torch.float32:
            raise RuntimeError("LayerNorm parameters must stay FP32")
        return self._hold(t.detach().contiguous())

    def _b32(self, model: "B200Transformer", name: str, b: torch.Tensor) -> int:
        src = model._bias_fp32.get(name)
        if src is None or src.shape != b.shape:
            src = b.detach()
        return self._hold(src.to(device=self.device, dtype=torch.float32).contiguous())

    def workspace(self, batch: int, seq: int):
        nbytes = ctypes.c_size_t()
        _lib.check(_lib.lib().tt_model_workspace_bytes(self.handle, batch, seq, ctypes.byref(nbytes)))
        return self._reserve(int(nbytes.value))

    def host_workspace(self, chunk: int, seq: int):
        nbytes = ctypes.c_size_t()
        _lib.check(_lib.lib().tt_model_host_workspace_bytes(self.handle, chunk, seq, ctypes.byref(nbytes)))
        return self._reserve(int(nbytes.value))

    def _reserve(self, need: int):
        """The workspace, grown to ``need`` bytes.  It is the library's own cudaMalloc
        (tt_workspace_alloc), not a PyTorch tensor: a forward first run inside a CUDA-graph
        warm-up (torch.compile(mode="reduce-overhead")) must not leave a live allocation in
        the graph's memory pool."""
        if self._ws_bytes < need:
            with torch.cuda.device(self.device):
                torch.cuda.current_stream(self.device).synchronize()  # the old one may be in use
                self._free_ws()
                ptr = ctypes.c_void_p()
                _lib.check(_lib.lib().tt_workspace_alloc(need + 1024, ctypes.byref(ptr)))
            self._ws_raw = ptr.value
            self._ws_ptr = (ptr.value + 1023) // 1024 * 1024
            self._ws_bytes = need + 1024 - (self._ws_ptr - ptr.value)
        return self._ws_ptr, self._ws_bytes

    def _free_ws(self) -> None:
        raw = getattr(self, "_ws_raw", 0)
        if raw:
            _lib.lib().tt_workspace_free(raw)
        self._ws_raw = 0
        self._ws_ptr = 0
        self._ws_bytes = 0

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            try:
                with torch.cuda.device(self.device):
                    torch.cuda.current_stream(self.device).synchronize()
                    self._free_ws()
                _lib.lib().tt_model_destroy(self.handle)
            except Exception:  # pragma: no cover - interpreter teardown
                pass
            self.handle = ctypes.c_void_p()

    def __del__(self) -> None:  # pragma: no cover
        self.close()


class B200Transformer(nn.Module):
    """FP16 tensor-core projections/attention, FP32 residual stream, LayerNorm and GELU.

    Drop-in for ``MixedPrecisionTransformer`` (mixed_precision/transformer.py:327-699):
    same ``__init__`` signature, module tree and parameter names; the enable_*
    switches are accepted for compatibility (the fused route is always used).
    """

    def __init__(
        self,
        config,
        *,
        enable_case11_schedule: bool = True,
        enable_attention_output_norm_fusion: bool = True,
        enable_full_ffn_fusion: bool = True,
        enable_fp16_custom_attention: bool = True,
        enable_fp16_normalized_stream: bool = True,
    ) -> None:
        super().__init__()
        self.config = config
        # Route flags the reference runner prints (mixed_precision_benchmark.py:67-77).
        # The reference's Triton routes do not exist here; these describe the B200 route.
        self.use_case8_triton = False
        self.use_d128_triton = False
        self.use_d32_triton = False
        self.use_d128_custom_attention = False
        self.use_case11_schedule = False
        self.use_fp16_custom_attention = True
        self.fuse_attention_output_norm = True
        self.fuse_full_ffn = False
        self.use_fp16_normalized_stream = True
        self.layers = nn.ModuleList(
            [
                MixedPrecisionTransformerBlock(config.d_model, config.num_heads, config.ffn_dim)
                for _ in range(config.num_layers)
            ]
        )
        self.final_norm = nn.LayerNorm(config.d_model)
        self.assume_all_tokens_valid = False
        self._bias_fp32: Dict[str, torch.Tensor] = {}
        self._plans: Dict[str, _DevicePlan] = {}
        self._op_key = _register(self)

    def __deepcopy__(self, memo):
        # Device plans hold C handles and are rebuilt on first use; the copy gets its own op key.
        cls = self.__class__
        new = cls.__new__(cls)
        memo[id(self)] = new
        for k, v in self.__dict__.items():
            new.__dict__[k] = {} if k == "_plans" else copy.deepcopy(v, memo)
        new._op_key = _register(new)
        return new

    # -- reference surface ---------------------------------------------------
    def convert_projections_to_fp16(self) -> None:
        """Linear weights and biases to FP16, as the reference does (transformer.py:476-478).

        The FP32 biases are kept aside first so the kernels can add them in
        full precision; LayerNorm parameters stay FP32.
        """
        for i, layer in enumerate(self.layers):
            for name, lin in (
                ("attention.qkv_proj", layer.attention.qkv_proj),
                ("attention.out_proj", layer.attention.out_proj),
                ("ffn_in", layer.ffn_in),
                ("ffn_out", layer.ffn_out),
            ):
                if lin.bias is not None and lin.bias.dtype == torch.float32:
                    self._bias_fp32[f"layers.{i}.{name}"] = lin.bias.detach().clone()
            layer.convert_projections_to_fp16()
        self._drop_plans()

    def route_description(self, seq_len: Optional[int] = None) -> str:
        cfg = self.config
        return _lib.route_describe(cfg.d_model, cfg.num_heads, seq_len or cfg.seq_len, cfg.ffn_dim)

    # -- execution -------------------------------------------------------------
    def _weights_key(self):
        return tuple(p.data_ptr() for p in self.parameters()) + tuple(
            t.data_ptr() for t in self._bias_fp32.values()
        )

    def _drop_plans(self) -> None:
        for plan in self._plans.values():
            plan.close()
        self._plans = {}

    def _plan(self, device: torch.device) -> _DevicePlan:
        key = str(device)
        plan = self._plans.get(key)
        if plan is None or plan.key != self._weights_key():
            if plan is not None:
                plan.close()
            plan = _DevicePlan(self, device)
            self._plans[key] = plan
        return plan

    def _apply(self, fn, recurse=True):
        self._drop_plans()
        out = super()._apply(fn, recurse)
        self._bias_fp32 = {k: fn(v) for k, v in self._bias_fp32.items()}
        return out

    def set_profiling(self, enable: bool, device: Optional[torch.device] = None) -> None:
        """Record CUDA events around every kernel of later forwards on ``device``."""
        dev = torch.device(device) if device is not None else next(self.parameters()).device
        _lib.check(_lib.lib().tt_model_set_profiling(self._plan(dev).handle, int(enable)))

    def profile_collect(self, device: Optional[torch.device] = None) -> Dict[str, tuple]:
        """{kernel kind: (total device ms, launches)} since the previous collect."""
        dev = torch.device(device) if device is not None else next(self.parameters()).device
        n = len(_lib.KERNEL_KINDS)
        ms = (ctypes.c_float * n)()
        cnt = (ctypes.c_int * n)()
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().tt_model_profile_collect(self._plan(dev).handle, ms, cnt, n))
        return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(_lib.KERNEL_KINDS)}

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.dtype != torch.float32:
            raise ValueError("mixed candidate requires an FP32 input/residual stream")
        if not x.is_cuda:
            # Host tensors are computed on the model's GPU through the pipelined host path.
            return self.forward_host(x, valid_token_mask)
        if x.dim() != 3 or x.shape[-1] != self.config.d_model:
            raise ValueError(f"expected x of shape [B, S, {self.config.d_model}], got {tuple(x.shape)}")
        mask = None if self.assume_all_tokens_valid else valid_token_mask
        if mask is not None and tuple(mask.shape) != tuple(x.shape[:2]):
            raise ValueError(f"valid_token_mask must have shape {tuple(x.shape[:2])}, got {tuple(mask.shape)}")
        # One custom op (tt_b200::model_forward): opaque to torch.compile, its fake
        # implementation gives the output's shape, and a CUDA-graph capture of it
        # records only this library's kernel launches.
        return torch.ops.tt_b200.model_forward(x, mask, self._op_key)

    def _forward_device(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        """The body of tt_b200::model_forward: one tt_model_forward call on x's device."""
        B, S, _ = x.shape
        x = x.contiguous()
        out = torch.empty_like(x)
        if B == 0 or S == 0:
            return out
        plan = self._plan(x.device)
        mask_ptr = 0
        if mask is not None:
            mask8 = mask.to(device=x.device, dtype=torch.bool).contiguous().view(torch.uint8)
            mask_ptr = mask8.data_ptr()
        ws_ptr, ws_bytes = plan.workspace(B, S)
        with torch.cuda.device(x.device):
            stream = torch.cuda.current_stream(x.device).cuda_stream
            _lib.check(
                _lib.lib().tt_model_forward(
                    plan.handle, x.data_ptr(), mask_ptr, out.data_ptr(), B, S, ws_ptr, ws_bytes, stream
                )
            )
        return out

    def reserve_workspace(self, batch: int, seq: int, device: Optional[torch.device] = None) -> None:
        """Allocates the device workspace for ``batch`` x ``seq`` now and runs one forward of zeros,
        so that later calls of that size or smaller allocate nothing and set nothing up (what a
        CUDA-graph capture of the forward, e.g. torch.compile(mode="reduce-overhead"), needs)."""
        dev = torch.device(device) if device is not None else next(self.parameters()).device
        plan = self._plan(dev)
        plan.workspace(batch, seq)
        with torch.inference_mode():
            self._forward_device(torch.zeros(batch, seq, self.config.d_model, device=dev), None)


    def forward_gather(
        self,
        x: torch.Tensor,
        valid_token_mask: Optional[torch.Tensor],
        out: torch.Tensor,
        gather_dst: int = 0,
    ) -> torch.Tensor:
        """``forward`` of this GPU's batch slice into ``out``, then pushed to ``gather_dst``.

        ``gather_dst`` is a device address on another GPU (a ``PeerGatherBuffer``
        slice) or 0.  One ``tt_model_forward_gather`` call: the push runs on the
        copy engines while later work on the current stream computes; the next
        call's last layer waits for it before rewriting ``out``.  Call
        ``gather_wait`` before relying on the destination.
        """
        if x.dtype != torch.float32 or not x.is_cuda or x.dim() != 3 or x.shape[-1] != self.config.d_model:
            raise ValueError("forward_gather takes an FP32 CUDA tensor [B, S, d_model]")
        if out.shape != x.shape or out.dtype != torch.float32 or out.device != x.device or not out.is_contiguous():
            raise ValueError("out must be a contiguous FP32 tensor shaped like x on x's device")
        B, S, _ = x.shape
        mask = None if self.assume_all_tokens_valid else valid_token_mask
        x = x.contiguous()
        plan = self._plan(x.device)
        mask_ptr = 0
        if mask is not None:
            if mask.shape != (B, S):
                raise ValueError(f"valid_token_mask must have shape {(B, S)}, got {tuple(mask.shape)}")
            mask8 = mask.to(device=x.device, dtype=torch.bool).contiguous().view(torch.uint8)
            mask_ptr = mask8.data_ptr()
        ws_ptr, ws_bytes = plan.workspace(B, S)
        with torch.cuda.device(x.device):
            stream = torch.cuda.current_stream(x.device).cuda_stream
            _lib.check(_lib.lib().tt_model_forward_gather(plan.handle, x.data_ptr(), mask_ptr, out.data_ptr(),
                                                          gather_dst or None, B, S, ws_ptr, ws_bytes, stream))
        return out

    def gather_wait(self, device: Optional[torch.device] = None) -> None:
        """Makes the current stream wait for every push ``forward_gather`` issued on ``device``."""
        dev = torch.device(device) if device is not None else next(self.parameters()).device
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
            _lib.check(_lib.lib().tt_model_gather_wait(self._plan(dev).handle, stream))

    def forward_host(
        self,
        x: torch.Tensor,
        valid_token_mask: Optional[torch.Tensor] = None,
        *,
        out: Optional[torch.Tensor] = None,
        chunk: Optional[int] = None,
        chunks: Optional[Sequence[int]] = None,
    ) -> torch.Tensor:
        """``forward`` for host tensors, on the GPU holding the model's parameters.

        One ``tt_model_forward_host`` call: the batch is cut into chunks of
        ``chunk`` sequences, and the copy-in of the next chunk and the copy-out
        of the previous one overlap the current chunk's kernels.  ``chunks``
        gives the schedule explicitly instead (sizes of consecutive chunks,
        adding up to the batch; ``tt_model_forward_host_chunks``).  ``x`` (and
        ``out``, when given) should be pinned; pageable tensors are staged
        through a pinned copy.  Returns ``out`` (a new pinned FP32 tensor when
        none is given) once the result is in host memory.
        """
        if x.dtype != torch.float32:
            raise ValueError("mixed candidate requires an FP32 input/residual stream")
        if x.is_cuda:
            raise ValueError("forward_host takes host tensors; use forward for CUDA tensors")
        dev = next(self.parameters()).device
        if dev.type != "cuda":
            raise RuntimeError("B200Transformer runs only on CUDA (sm_100a) devices; there is no CPU path")
        if x.dim() != 3 or x.shape[-1] != self.config.d_model:
            raise ValueError(f"expected x of shape [B, S, {self.config.d_model}], got {tuple(x.shape)}")
        B, S, _ = x.shape
        x = x.contiguous()
        if not x.is_pinned():
            x = x.pin_memory()
        if out is None:
            out = torch.empty(x.shape, dtype=torch.float32, pin_memory=True)
        elif out.shape != x.shape or out.dtype != torch.float32 or out.is_cuda or not out.is_contiguous():
            # (the library itself rejects pageable memory: out may also be host memory that was
            # page-locked with cudaHostRegister, which torch does not always report as pinned)
            raise ValueError("out must be a contiguous page-locked FP32 host tensor shaped like x")
        if B == 0 or S == 0:
            return out
        mask = None if self.assume_all_tokens_valid else valid_token_mask
        mask_ptr = 0
        if mask is not None:
            if mask.shape != (B, S):
                raise ValueError(f"valid_token_mask must have shape {(B, S)}, got {tuple(mask.shape)}")
            mask8 = mask.to(device="cpu", dtype=torch.bool).contiguous().view(torch.uint8)
            if not mask8.is_pinned():
                mask8 = mask8.pin_memory()
            mask_ptr = mask8.data_ptr()
        plan = self._plan(dev)
        if chunks is not None:
            sizes = [int(c) for c in chunks]
            if not sizes or min(sizes) <= 0 or sum(sizes) != B:
                raise ValueError(f"chunks must be positive sizes adding up to the batch {B}, got {sizes}")
            ws_ptr, ws_bytes = plan.host_workspace(max(sizes), S)
            arr = (ctypes.c_int * len(sizes))(*sizes)
        else:
            if chunk is None:
                chunk = default_host_chunk(B, S, self.config.d_model)
            chunk = max(1, min(int(chunk), B))
            ws_ptr, ws_bytes = plan.host_workspace(chunk, S)
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev)
            if chunks is not None:
                rc = _lib.lib().tt_model_forward_host_chunks(
                    plan.handle, x.data_ptr(), mask_ptr, out.data_ptr(), B, S, arr, len(sizes), ws_ptr, ws_bytes,
                    stream.cuda_stream,
                )
            else:
                rc = _lib.lib().tt_model_forward_host(
                    plan.handle, x.data_ptr(), mask_ptr, out.data_ptr(), B, S, chunk, ws_ptr, ws_bytes,
                    stream.cuda_stream,
                )
            _lib.check(rc)
            stream.synchronize()
        return out


    def capture_graph(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> "GraphedForward":
        """Captures one forward over ``x`` as a CUDA graph (``tt_model_graph_create``).

        Returns a callable that replays it: write new inputs into
        ``graphed.x`` (same shape), call ``graphed()``, read ``graphed.out``.
        The graph owns its workspace and output; the model stays usable for
        ordinary calls.
        """
        if x.dtype != torch.float32 or not x.is_cuda or x.dim() != 3 or x.shape[-1] != self.config.d_model:
            raise ValueError("capture_graph takes an FP32 CUDA tensor [B, S, d_model]")
        return GraphedForward(self, x, None if self.assume_all_tokens_valid else valid_token_mask)


class GraphedForward:
    """A captured forward: static input ``x``, static output ``out``, one graph replay per call."""

    def __init__(self, model: B200Transformer, x: torch.Tensor, mask: Optional[torch.Tensor]) -> None:
        B, S, _ = x.shape
        self.x = x.contiguous()
        self.out = torch.empty_like(self.x)
        self.mask = None
        mask_ptr = 0
        if mask is not None:
            if mask.shape != (B, S):
                raise ValueError(f"valid_token_mask must have shape {(B, S)}, got {tuple(mask.shape)}")
            self.mask = mask.to(device=x.device, dtype=torch.bool).contiguous().view(torch.uint8)
            mask_ptr = self.mask.data_ptr()
        self.device = x.device
        self._plan = model._plan(x.device)
        nbytes = ctypes.c_size_t()
        _lib.check(_lib.lib().tt_model_workspace_bytes(self._plan.handle, B, S, ctypes.byref(nbytes)))
        raw = torch.empty(int(nbytes.value) + 1024, dtype=torch.uint8, device=x.device)
        self._ws = raw
        ws_ptr = (raw.data_ptr() + 1023) // 1024 * 1024
        handle = ctypes.c_void_p()
        with torch.cuda.device(x.device):
            torch.cuda.current_stream(x.device).synchronize()
            _lib.check(_lib.lib().tt_model_graph_create(
                self._plan.handle, self.x.data_ptr(), mask_ptr, self.out.data_ptr(), B, S, ws_ptr,
                int(nbytes.value), ctypes.byref(handle)))
        self._handle = handle

    def __call__(self) -> torch.Tensor:
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _lib.check(_lib.lib().tt_graph_launch(self._handle, stream))
        return self.out

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            try:
                _lib.lib().tt_graph_destroy(self._handle)
            except Exception:  # pragma: no cover - interpreter teardown
                pass
            self._handle = ctypes.c_void_p()

    def __del__(self) -> None:  # pragma: no cover
        self.close()


# ---------------------------------------------------------------- the custom op
# Models are reached from the op by an integer key (the op's arguments can only be
# tensors and scalars); the registry holds weak references.
_REGISTRY: Dict[int, "weakref.ReferenceType[B200Transformer]"] = {}
_KEYS = itertools.count(1)


def _register(model: "B200Transformer") -> int:
    key = next(_KEYS)
    _REGISTRY[key] = weakref.ref(model)
    return key


@torch.library.custom_op("tt_b200::model_forward", mutates_args=())
def _model_forward_op(x: torch.Tensor, mask: Optional[torch.Tensor], key: int) -> torch.Tensor:
    """FP32 [B, S, D] -> FP32 [B, S, D]: the whole forward (tt_model_forward) of the model registered as key."""
    ref = _REGISTRY.get(key)
    model = ref() if ref is not None else None
    if model is None:
        raise RuntimeError(f"tt_b200::model_forward: no live model under key {key}")
    return model._forward_device(x, mask)


@_model_forward_op.register_fake
def _(x: torch.Tensor, mask: Optional[torch.Tensor], key: int) -> torch.Tensor:
    return torch.empty_like(x, memory_format=torch.contiguous_format)


def default_host_chunk(batch: int, seq: int, d_model: int) -> int:
    """Sequences per chunk of the host pipeline: up to 8 chunks of at least 8 MiB of input each."""
    total = batch * seq * d_model * 4
    n_chunks = max(1, min(8, total // (8 << 20), batch))
    return (batch + n_chunks - 1) // n_chunks


# The reference's class name, for drop-in imports.
MixedPrecisionTransformer = B200Transformer


def copy_mixed_model_weights(baseline: nn.Module, mixed: nn.Module) -> None:
    """Copy FP32 baseline weights into the mixed model, packing Q/K/V.

    Same contract as mixed_precision/transformer.py:702-731: for every
    ``attention.qkv_proj`` tensor the baseline's q/k/v tensors are
    concatenated along dim 0; everything else is copied by name; strict load.
    """
    source = copy.deepcopy(baseline.state_dict())
    mapped = {}
    for key in mixed.state_dict():
        for leaf in ("weight", "bias"):
            suffix = f"attention.qkv_proj.{leaf}"
            if key.endswith(suffix):
                prefix = key[: -len(suffix)] + "attention."
                mapped[key] = torch.cat(
                    [source[f"{prefix}{n}_proj.{leaf}"] for n in ("q", "k", "v")], dim=0
                )
                break
        else:
            mapped[key] = source[key]
    mixed.load_state_dict(mapped, strict=True)


class PreallocatedMicrobatchModel(nn.Module):
    """Runs ``model`` over microbatches of ``microbatch_size`` sequences into one preallocated output.

    Same contract as the reference runner's wrapper (mixed_precision_benchmark.py:13-33),
    which it applies automatically to batches of 4096 or more (:79-84): a batch no
    larger than one microbatch goes straight to ``model``; otherwise every slice of
    ``x`` (and of the mask) runs separately and is copied into an FP32 output shaped
    like ``x``.  A B200Transformer needs no microbatching for memory (its whole batch
    runs as one call); the wrapper is here so that runners which apply it keep working.
    """

    def __init__(self, model: nn.Module, microbatch_size: int) -> None:
        super().__init__()
        if microbatch_size <= 0:
            raise ValueError("microbatch_size must be positive")
        self.model = model
        self.microbatch_size = microbatch_size

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.shape[0] <= self.microbatch_size:
            return self.model(x, valid_token_mask)
        output = torch.empty_like(x, dtype=torch.float32)
        for start in range(0, x.shape[0], self.microbatch_size):
            end = min(start + self.microbatch_size, x.shape[0])
            mask_slice = None if valid_token_mask is None else valid_token_mask[start:end]
            output[start:end].copy_(self.model(x[start:end], mask_slice))
        return output
