"""Drop-in `UserOptimizedTransformer` on the B200 C-ABI library.

Public surface follows v16_1_clean.py:376-735: the constructor takes a config
exposing batch_size, seq_len, d_model, num_heads, ffn_dim, num_layers, causal
and validate(); the parameter tree and strict state_dict are the reference's
(`layers.{i}.norm1`, `.attention.{q,k,v,out}_proj`, `.norm2`, `.ffn_in`,
`.ffn_out`, `final_norm`; torch_transformer_benchmark.py:148-160 and
v16_1_clean.py:76-134,385-406); fp16 weight caches are non-persistent buffers
rebuilt on load_state_dict/_apply (v16_1_clean.py:412-464).

forward(x [B,S,D] fp32 CUDA, valid_token_mask [B,S] bool or None) runs the
whole encoder as one tj_encoder_forward call on the current stream: token
plan, then per layer LN1->fp16, QKV GEMM (head-major), flash attention,
out-proj (fp16), residual add + LN2->fp16, FFN-in+GELU, FFN-out (fp16), and
the residual add fused into the next layer's LN1 or the final LayerNorm,
which scatters back to [B,S,D] with padded rows zeroed.  There is no eager or
CPU fallback: a CPU tensor, a non-fp32 input, training mode or a missing
library raises.
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, Optional

import torch
import torch.nn as nn

from . import _lib

__all__ = ["TransformerConfig", "UserOptimizedTransformer"]


@dataclass(frozen=True)
class TransformerConfig:
    """Same fields and checks as v16_1_clean.py:49-73."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")


class _SelfAttention(nn.Module):
    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim**-0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)
        # Non-persistent caches (v16_1_clean.py:92-103): packed fp16 QKV weight,
        # fp32 packed QKV bias (added to the fp32 accumulator), fp16 out weight.
        self.register_buffer("_qkv_weight_mixed", torch.empty(0), persistent=False)
        self.register_buffer("_qkv_bias_mixed", torch.empty(0), persistent=False)
        self.register_buffer("_out_weight_mixed", torch.empty(0), persistent=False)


class _TransformerBlock(nn.Module):
    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = _SelfAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)
        self.register_buffer("_ffn_in_weight_mixed", torch.empty(0), persistent=False)
        self.register_buffer("_ffn_out_weight_mixed", torch.empty(0), persistent=False)


class UserOptimizedTransformer(nn.Module):
    """B200 (sm_100a) encoder with the reference's API and state_dict."""

    internal_dtype = torch.float16
    _LARGE_SEQUENCE_CUTOFF = 8_192
    _LARGE_SEQUENCE_BATCH_CHUNK = 1

    def __init__(self, config: Any) -> None:
        super().__init__()
        config.validate()
        self.config = config
        self.layers = nn.ModuleList(
            [_TransformerBlock(config.d_model, config.num_heads, config.ffn_dim) for _ in range(config.num_layers)]
        )
        self.final_norm = nn.LayerNorm(config.d_model)
        self._large_sequence_compile_enabled = True
        self._large_sequence_compile_backend: Optional[str] = None
        self._large_sequence_compile_mode: Optional[str] = "max-autotune"
        self._large_sequence_compile_fullgraph = False
        self.__dict__["_workspace"] = None
        self.__dict__["_layer_structs"] = None
        self.__dict__["_graphs"] = OrderedDict()
        self.use_cuda_graphs = True
        self._refresh_mixed_weights()

    # ---- weight caches ------------------------------------------------------
    @staticmethod
    def _cast_cache(t: torch.Tensor) -> torch.Tensor:
        """fp16 copy of an [N, K] weight with rows padded by zeros to a multiple
        of 8 columns (whole 16-byte rows for the GEMM's TMA loads; the encoder
        reads only the first K)."""
        w = t.detach().to(dtype=torch.float16)
        pad = -w.shape[1] % 8
        if pad:
            w = torch.nn.functional.pad(w, (0, pad))
        return w.contiguous()

    def _refresh_mixed_weights(self) -> None:
        """Rebuilds the fp16 caches (v16_1_clean.py:412-442)."""
        for layer in self.layers:
            att = layer.attention
            att._qkv_weight_mixed = self._cast_cache(
                torch.cat((att.q_proj.weight, att.k_proj.weight, att.v_proj.weight))
            )
            att._qkv_bias_mixed = torch.cat((att.q_proj.bias, att.k_proj.bias, att.v_proj.bias)).detach().float().contiguous()
            att._out_weight_mixed = self._cast_cache(att.out_proj.weight)
            layer._ffn_in_weight_mixed = self._cast_cache(layer.ffn_in.weight)
            layer._ffn_out_weight_mixed = self._cast_cache(layer.ffn_out.weight)
        self.__dict__["_layer_structs"] = None
        self._drop_graphs()

    def load_state_dict(self, state_dict, *args, **kwargs):
        result = super().load_state_dict(state_dict, *args, **kwargs)
        self._refresh_mixed_weights()
        return result

    def _apply(self, fn, recurse: bool = True):
        result = super()._apply(fn, recurse=recurse)
        self._refresh_mixed_weights()
        self.__dict__["_workspace"] = None
        return result

    # ---- large-sequence API of the reference (v16_1_clean.py:630-726) -------
    # API compatibility shims.  The reference bounds memory for B>1, S>=8192
    # with a per-sample loop around a torch.compile'd executor.  Here attention
    # is a flash kernel (O(S) memory) for every shape, so these entry points
    # run the native path: configure_large_sequence_executor only records its
    # arguments (nothing reads them; there is no compiled executor), and
    # large_sequence_executor_ready is always True.
    def _uses_large_sequence_chunking(self, x: torch.Tensor) -> bool:
        return (
            not self.training
            and x.dtype == torch.float32
            and x.ndim == 3
            and x.shape[0] > 1
            and x.shape[1] >= self._LARGE_SEQUENCE_CUTOFF
        )

    def configure_large_sequence_executor(self, *, enabled: bool = True, backend: Optional[str] = None,
                                          mode: Optional[str] = "max-autotune", fullgraph: bool = False) -> None:
        if backend is not None and mode is not None and backend != "inductor":
            raise ValueError("mode must be None for non-Inductor backends")
        self._large_sequence_compile_enabled = enabled
        self._large_sequence_compile_backend = backend
        self._large_sequence_compile_mode = mode
        self._large_sequence_compile_fullgraph = fullgraph

    @property
    def large_sequence_executor_ready(self) -> bool:
        return True

    def prepare_large_sequence_executor(self):
        if self.training:
            raise RuntimeError("large-sequence executor requires eval mode")
        return self._forward_impl

    def forward_large_sequence_sample(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.training or x.dtype != torch.float32:
            raise ValueError("compiled sample path requires FP32 eval mode")
        if x.ndim != 3 or x.shape[0] != 1:
            raise ValueError("compiled sample path requires shape [1,S,D]")
        if x.shape[1] < self._LARGE_SEQUENCE_CUTOFF:
            raise ValueError("sequence length is below the large-sequence cutoff")
        if valid_token_mask is not None and valid_token_mask.shape != x.shape[:2]:
            raise ValueError("valid_token_mask must have shape [1,S]")
        return self._forward_impl(x, valid_token_mask)

    # ---- forward -------------------------------------------------------------
    def _layer_weights(self, device: torch.device):
        structs = self.__dict__.get("_layer_structs")
        if structs is not None and structs[0] == device:
            return structs[1]
        arr = (_lib.LayerWeights * len(self.layers))()
        for i, layer in enumerate(self.layers):
            att = layer.attention
            tensors = [
                layer.norm1.weight, layer.norm1.bias, att._qkv_weight_mixed, att._qkv_bias_mixed,
                att._out_weight_mixed, att.out_proj.bias, layer.norm2.weight, layer.norm2.bias,
                layer._ffn_in_weight_mixed, layer.ffn_in.bias, layer._ffn_out_weight_mixed, layer.ffn_out.bias,
            ]
            for t in tensors:
                if t.device != device:
                    raise ValueError(f"model parameters are on {t.device}, input is on {device}; call .to({device})")
                if not t.is_contiguous():
                    raise ValueError("model parameters must be contiguous")
            f = arr[i]
            (f.ln1_gamma, f.ln1_beta, f.w_qkv16, f.b_qkv, f.w_out16, f.b_out, f.ln2_gamma, f.ln2_beta,
             f.w_ffn_in16, f.b_ffn_in, f.w_ffn_out16, f.b_ffn_out) = [t.data_ptr() for t in tensors]
        self.__dict__["_layer_structs"] = (device, arr)
        return arr

    def _workspace_for(self, desc: "_lib.EncoderDesc", device: torch.device) -> torch.Tensor:
        lib = _lib.load()
        need = lib.tj_encoder_workspace_bytes(ctypes.byref(desc))
        if need <= 0:
            raise ValueError("invalid encoder shape")
        ws = self.__dict__.get("_workspace")
        if ws is None or ws.device != device or ws.numel() < need:
            self._drop_graphs()  # captured graphs point at the old workspace
            ws = torch.empty(need, dtype=torch.uint8, device=device)
            self.__dict__["_workspace"] = ws
        return ws

    def _check_inputs(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]):
        if self.training:
            raise RuntimeError("UserOptimizedTransformer runs inference only; call .eval()")
        if not isinstance(x, torch.Tensor) or x.ndim != 3:
            raise ValueError("x must be a [batch, seq_len, d_model] tensor")
        if x.dtype != torch.float32:
            raise TypeError(f"x must be float32, got {x.dtype}")
        if x.device.type != "cuda":
            raise ValueError("x must be a CUDA tensor (the library has no CPU path)")
        if x.requires_grad:
            raise RuntimeError("autograd through the encoder is not supported")
        if x.shape[-1] != self.config.d_model:
            raise ValueError(f"x last dimension {x.shape[-1]} != d_model {self.config.d_model}")
        mask = None
        if valid_token_mask is not None:
            if valid_token_mask.shape != x.shape[:2]:
                raise ValueError(f"valid_token_mask must have shape {tuple(x.shape[:2])}")
            if valid_token_mask.dtype not in (torch.bool, torch.uint8):
                raise TypeError("valid_token_mask must be bool")
            if valid_token_mask.device != x.device:
                raise ValueError("valid_token_mask must be on the same device as x")
            mask = valid_token_mask.contiguous()
            if mask.dtype == torch.bool:
                mask = mask.view(torch.uint8)
        return x.contiguous(), mask

    def _launch(self, x: torch.Tensor, mask: Optional[torch.Tensor], out: torch.Tensor) -> None:
        """One tj_encoder_forward call on the current stream."""
        B, S, D = x.shape
        cfg = self.config
        desc = _lib.EncoderDesc(B, S, D, cfg.num_heads, cfg.ffn_dim, len(self.layers), 1 if cfg.causal else 0,
                                float(self.final_norm.eps))
        lib = _lib.load()
        ws = self._workspace_for(desc, x.device)
        weights = self._layer_weights(x.device)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        rc = lib.tj_encoder_forward(
            ctypes.byref(desc), weights, self.final_norm.weight.data_ptr(), self.final_norm.bias.data_ptr(),
            x.data_ptr(), None if mask is None else mask.data_ptr(), out.data_ptr(), ws.data_ptr(),
            ws.numel(), ctypes.c_void_p(stream),
        )
        _lib.check(rc, "encoder_forward")

    # ---- CUDA graphs for small problems -------------------------------------
    # Each kernel launch costs a few microseconds of host work (argument checks,
    # tensor-map encoding, the launch itself).  A small problem's whole forward
    # takes about that long per kernel on the GPU, so the GPU would wait for
    # the host.  For inputs up to _GRAPH_MAX_INPUT_BYTES the forward of each
    # input shape is captured once into a CUDA graph over static input, mask
    # and output buffers; a call copies its input in, replays the graph and
    # returns a copy of the output (so later calls never alias it).
    _GRAPH_MAX_INPUT_BYTES = 32 << 20
    _GRAPH_CACHE_SIZE = 8

    def _drop_graphs(self) -> None:
        graphs = self.__dict__.get("_graphs")
        if graphs:
            graphs.clear()

    def _graph_forward(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        dev = x.device
        stream = torch.cuda.current_stream(dev)
        key = (dev, tuple(x.shape), mask is None, stream.cuda_stream)
        graphs = self.__dict__["_graphs"]
        entry = graphs.get(key)
        if entry is None:
            sx = torch.empty_like(x)
            sm = None if mask is None else torch.empty_like(mask)
            so = torch.empty_like(x)
            sx.copy_(x)
            if sm is not None:
                sm.copy_(mask)
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):  # warm-up: kernel attributes, workspace
                self._launch(sx, sm, so)
            stream.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._launch(sx, sm, so)
            entry = (graph, sx, sm, so)
            graphs[key] = entry
            while len(graphs) > self._GRAPH_CACHE_SIZE:
                graphs.popitem(last=False)
        else:
            graphs.move_to_end(key)
        graph, sx, sm, so = entry
        sx.copy_(x)
        if sm is not None:
            sm.copy_(mask)
        graph.replay()
        return so.clone()

    def _forward_impl(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
        x, mask = self._check_inputs(x, valid_token_mask)
        if x.shape[0] == 0 or x.shape[1] == 0:
            return torch.empty_like(x)  # an empty batch, as the eager model returns
        if (self.use_cuda_graphs and x.numel() * 4 <= self._GRAPH_MAX_INPUT_BYTES
                and not _lib.sync_check_enabled()
                and not torch.cuda.is_current_stream_capturing()):
            return self._graph_forward(x, mask)
        out = torch.empty_like(x)
        self._launch(x, mask, out)
        return out

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self._forward_impl(x, valid_token_mask)
