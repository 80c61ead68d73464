"""``B200Stage``: one pipeline stage whose weights, KV cache and kernels live
in the C-ABI library.

The Python object keeps the reference stage's public surface — ``cfg``,
``layer_start`` / ``layer_end``, ``has_embedding`` / ``has_lm_head``,
``cache_length`` / ``trim_cache`` — and its argument validation with the same
messages (models/llama_dense.py:375-481), then hands device pointers to
``mg_stage_forward``.  Nothing here computes: every operation on activations
runs in the library's CUDA kernels.
"""
from __future__ import annotations

import ctypes
from typing import Any, NamedTuple

import torch

from gpu_mesh_b200 import _lib
from gpu_mesh_b200.config import LlamaConfig, config_from
from gpu_mesh_b200.weights import rope_tables

_DTYPES = {torch.float32: _lib.MG_DTYPE_F32, torch.bfloat16: _lib.MG_DTYPE_BF16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _DeviceArray:
    """A device pointer as ``__cuda_array_interface__`` (torch wraps it without a copy)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3, "strides": None,
        }


class _LoadResult(NamedTuple):
    missing_keys: list[str]
    unexpected_keys: list[str]


class _Submodule:
    """A named part of the stage (``embed_tokens``, ``norm``, ``lm_head``,
    ``layers[i]``) with the nn.Module weight methods callers use on the
    reference's LlamaStage submodules, over the stage's own HBM views."""

    def __init__(self, stage: "B200Stage", prefix: str) -> None:
        self._stage, self._prefix = stage, prefix + "."

    def named_parameters(self):
        n = len(self._prefix)
        for k, v in self._stage.named_parameters():
            if k.startswith(self._prefix):
                yield k[n:], v

    def parameters(self):
        for _, v in self.named_parameters():
            yield v

    def state_dict(self) -> dict[str, torch.Tensor]:
        n = len(self._prefix)
        return {k[n:]: v for k, v in self._stage.state_dict().items() if k.startswith(self._prefix)}

    def load_state_dict(self, state_dict: dict[str, torch.Tensor], strict: bool = True):
        own = self.state_dict()
        missing = [k for k in own if k not in state_dict]
        unexpected = [k for k in state_dict if k not in own]
        if strict and (missing or unexpected):
            raise RuntimeError(f"Error(s) in loading state_dict for {self._prefix[:-1]}: missing keys "
                               f"{missing}, unexpected keys {unexpected}")
        full = {self._prefix + k: v for k, v in state_dict.items() if k in own}
        self._stage.load_state_dict(full, strict=False)
        return _LoadResult(missing, unexpected)


class B200Stage:
    """Contiguous decoder layers [layer_start, layer_end) on one B200.

    ``state_dict`` uses the reference stage's key names (local layer indices);
    tensors may live on any device and are copied into the stage's own HBM
    layout, after which the caller may drop them.
    """

    supports_cache_flag = True

    def __init__(
        self,
        cfg: Any,
        layer_start: int,
        layer_end: int,
        *,
        has_embedding: bool = False,
        has_lm_head: bool = False,
        device: torch.device | str | int = "cuda",
        dtype: torch.dtype = torch.bfloat16,
        state_dict: dict[str, torch.Tensor],
    ) -> None:
        cfg = config_from(cfg)
        if not 0 <= layer_start < layer_end <= cfg.num_hidden_layers:
            raise ValueError(
                f"invalid layer range [{layer_start}, {layer_end}) for "
                f"{cfg.num_hidden_layers} layers"
            )
        if dtype not in _DTYPES:
            raise ValueError(f"unsupported stage dtype {dtype}; use torch.float32 or torch.bfloat16")
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("a B200 stage runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.cfg = cfg
        self.layer_start = layer_start
        self.layer_end = layer_end
        self.has_embedding = has_embedding
        self.has_lm_head = has_lm_head
        self.device = device
        self.dtype = dtype
        self._handle = ctypes.c_void_p()
        self._lib = _lib.lib()

        def get(key: str, required: bool = True) -> torch.Tensor | None:
            t = state_dict.get(key)
            if t is None:
                if required:
                    raise KeyError(f"state_dict is missing {key!r}")
                return None
            return t.detach().to(device=device, dtype=dtype).contiguous()

        keep: list[torch.Tensor] = []

        def hold(t: torch.Tensor | None) -> int | None:
            if t is not None:
                keep.append(t)
            return _ptr(t)

        n_local = layer_end - layer_start
        layers = (_lib.LayerWeights * n_local)()
        for i in range(n_local):
            p = f"layers.{i}."
            lw = layers[i]
            lw.input_layernorm = hold(get(p + "input_layernorm.weight"))
            lw.q_proj = hold(get(p + "self_attn.q_proj.weight"))
            lw.k_proj = hold(get(p + "self_attn.k_proj.weight"))
            lw.v_proj = hold(get(p + "self_attn.v_proj.weight"))
            lw.o_proj = hold(get(p + "self_attn.o_proj.weight"))
            lw.q_norm = hold(get(p + "self_attn.q_norm.weight", cfg.qk_norm)) if cfg.qk_norm else None
            lw.k_norm = hold(get(p + "self_attn.k_norm.weight", cfg.qk_norm)) if cfg.qk_norm else None
            lw.post_attention_layernorm = hold(get(p + "post_attention_layernorm.weight"))
            lw.gate_proj = hold(get(p + "mlp.gate_proj.weight"))
            lw.up_proj = hold(get(p + "mlp.up_proj.weight"))
            lw.down_proj = hold(get(p + "mlp.down_proj.weight"))
        cos, sin = rope_tables(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta, dtype,
                               round_inv_freq=cfg.mask_policy == "cache")
        weights = _lib.StageWeights()
        weights.rope_cos = hold(cos.to(device))
        weights.rope_sin = hold(sin.to(device))
        weights.layers = layers
        if has_embedding:
            weights.embed_tokens = hold(get("embed_tokens.weight"))
        if has_lm_head:
            weights.norm = hold(get("norm.weight"))
            head = state_dict.get("lm_head.weight")
            embed = state_dict.get("embed_tokens.weight")
            if has_embedding and head is not None and embed is not None and head is embed:
                weights.lm_head = weights.embed_tokens  # tied: share the stage copy
            else:
                weights.lm_head = hold(get("lm_head.weight"))

        c = _lib.StageConfig()
        c.vocab_size = cfg.vocab_size
        c.hidden_size = cfg.hidden_size
        c.intermediate_size = cfg.intermediate_size
        c.num_hidden_layers = cfg.num_hidden_layers
        c.num_attention_heads = cfg.num_attention_heads
        c.num_key_value_heads = cfg.num_key_value_heads
        c.head_dim = cfg.head_dim
        c.max_position_embeddings = cfg.max_position_embeddings
        c.rms_norm_eps = cfg.rms_norm_eps
        c.qk_norm = int(cfg.qk_norm)
        c.attention_impl = cfg.attention_impl_code
        c.dtype = _DTYPES[dtype]
        c.layer_start = layer_start
        c.layer_end = layer_end
        c.has_embedding = int(has_embedding)
        c.has_lm_head = int(has_lm_head)
        c.device = device.index
        torch.cuda.synchronize(device)
        _lib.check(self._lib.mg_stage_create(ctypes.byref(c), ctypes.byref(weights), ctypes.byref(self._handle)))
        torch.cuda.synchronize(device)
        del keep

    # ------------------------------------------------------------------
    def close(self) -> None:
        if self._handle:
            self._lib.mg_stage_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._handle:
            raise RuntimeError("stage has been closed")
        return self._handle

    def memory(self) -> dict[str, int]:
        w, k, x = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        _lib.check(self._lib.mg_stage_memory(self.handle, ctypes.byref(w), ctypes.byref(k), ctypes.byref(x)))
        return {"weights": w.value, "kv": k.value, "work": x.value}

    # ------------------------------------------------------------------
    # KV slots
    # ------------------------------------------------------------------
    def kv_length(self, slot: int) -> int:
        n = ctypes.c_int32()
        _lib.check(self._lib.mg_kv_length(self.handle, slot, ctypes.byref(n)))
        return n.value

    def kv_batch(self, slot: int) -> int:
        n = ctypes.c_int32()
        _lib.check(self._lib.mg_kv_batch(self.handle, slot, ctypes.byref(n)))
        return n.value

    def kv_reserve(self, slot: int, batch: int, capacity: int) -> None:
        """Create an empty slot for `batch` rows and `capacity` positions."""
        _lib.check(self._lib.mg_kv_alloc(self.handle, slot, batch, capacity))

    def kv_free(self, slot: int) -> None:
        _lib.check(self._lib.mg_kv_free(self.handle, slot))

    def kv_free_all(self) -> None:
        _lib.check(self._lib.mg_kv_free_all(self.handle))

    def kv_trim(self, slot: int, length: int) -> None:
        _lib.check(self._lib.mg_kv_trim(self.handle, slot, length))

    def kv_import(self, slot: int, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Write [B, nkv, T, D] keys/values of one local layer into a slot."""
        k = k.to(device=self.device, dtype=self.dtype).contiguous()
        v = v.to(device=self.device, dtype=self.dtype).contiguous()
        if k.shape != v.shape or k.ndim != 4:
            raise ValueError("KV cache tensors must have matching shape [B, Hkv, S, D]")
        if k.shape[1] != self.cfg.num_key_value_heads or k.shape[3] != self.cfg.head_dim:
            raise ValueError("KV cache shape does not match model configuration")
        if self.kv_batch(slot) != k.shape[0]:
            self.kv_reserve(slot, k.shape[0], max(k.shape[2], 1))
        _lib.check(
            self._lib.mg_kv_import(self.handle, slot, layer, k.data_ptr(), v.data_ptr(), k.shape[2],
                                   _stream(self.device))
        )

    def kv_export(self, slot: int) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """The slot's cache as the reference's list of per-layer (k, v) tensors."""
        B, T = self.kv_batch(slot), self.kv_length(slot)
        out = []
        for layer in range(self.layer_end - self.layer_start):
            shape = (B, self.cfg.num_key_value_heads, T, self.cfg.head_dim)
            k = torch.empty(shape, dtype=self.dtype, device=self.device)
            v = torch.empty(shape, dtype=self.dtype, device=self.device)
            if B and T:
                _lib.check(
                    self._lib.mg_kv_export(self.handle, slot, layer, k.data_ptr(), v.data_ptr(),
                                           _stream(self.device))
                )
            out.append((k, v))
        return out

    # ------------------------------------------------------------------
    # Forward
    # ------------------------------------------------------------------
    def validate(
        self,
        x: torch.Tensor | None,
        input_ids: torch.Tensor | None,
        position_ids: torch.Tensor | None,
        past_len: int,
        *,
        check_values: bool = True,
    ) -> tuple[int, int, torch.Tensor | None]:
        """Argument checks of LlamaStage.forward (llama_dense.py:375-481).

        Returns (B, S, positions as int64 [B, S] on the device or None).
        """
        cfg = self.cfg
        if self.has_embedding:
            if input_ids is None:
                raise ValueError("the embedding stage requires input_ids")
            if input_ids.ndim != 2 or input_ids.shape[0] < 1 or input_ids.shape[1] < 1:
                raise ValueError("input_ids must have shape [batch, sequence] and be non-empty")
            if input_ids.dtype not in (torch.int32, torch.int64):
                raise ValueError("input_ids must use int32 or int64 dtype")
            if check_values:
                lo, hi = int(input_ids.min().item()), int(input_ids.max().item())
                if lo < 0 or hi >= cfg.vocab_size:
                    raise ValueError(f"input_ids contain a value outside [0, {cfg.vocab_size})")
            B, S = input_ids.shape
        else:
            if input_ids is not None:
                raise ValueError("input_ids are only accepted by the embedding stage")
            if x is None or x.ndim != 3 or x.shape[0] < 1 or x.shape[1] < 1:
                raise ValueError("a non-embedding stage requires non-empty hidden states [B, S, H]")
            if x.shape[-1] != cfg.hidden_size:
                raise ValueError(
                    f"hidden state width {x.shape[-1]} != model hidden_size {cfg.hidden_size}"
                )
            if x.dtype != self.dtype:
                raise ValueError(f"hidden states must use the stage dtype {self.dtype}, got {x.dtype}")
            B, S = x.shape[0], x.shape[1]

        pos = None
        if position_ids is not None:
            if position_ids.ndim != 2 or position_ids.shape[1] != S:
                raise ValueError("position_ids must have shape [batch or 1, sequence] matching input")
            if position_ids.shape[0] not in (1, B):
                raise ValueError("position_ids batch dimension must be 1 or input batch")
            if position_ids.dtype not in (torch.int32, torch.int64):
                raise ValueError("position_ids must use int32 or int64 dtype")
            pos = position_ids.to(device=self.device, dtype=torch.int64).expand(B, S).contiguous()
            if check_values:
                lo, hi = int(pos.min().item()), int(pos.max().item())
                if lo < 0 or hi >= cfg.max_position_embeddings:
                    raise ValueError(
                        "position_ids contain a value outside "
                        f"[0, {cfg.max_position_embeddings})"
                    )
        if past_len + S > cfg.max_position_embeddings:
            raise ValueError(
                f"sequence would reach {past_len + S} positions, "
                f"but model context is {cfg.max_position_embeddings}"
            )
        return B, S, pos

    def forward_slot(
        self,
        slot: int,
        x: torch.Tensor | None,
        *,
        input_ids: torch.Tensor | None = None,
        position_ids: torch.Tensor | None = None,
        logits: str = "all",
        check_values: bool = True,
    ) -> torch.Tensor:
        """Run the stage for one KV slot; appends this input to the slot's cache.

        ``logits="all"`` returns [B, S, V] like the reference; ``"last"`` only
        the final position [B, 1, V] (last stage only).
        """
        past = self.kv_length(slot)
        B, S, pos = self.validate(x, input_ids, position_ids, past, check_values=check_values)
        if past and self.kv_batch(slot) != B:
            raise ValueError("KV cache shape does not match model configuration")
        ids = None
        if input_ids is not None:
            ids = input_ids.to(device=self.device, dtype=torch.int64).contiguous()
        if x is not None and not self.has_embedding:
            x = x.to(self.device).contiguous()
        if self.has_lm_head:
            mode = _lib.MG_OUT_LOGITS_LAST if logits == "last" else _lib.MG_OUT_LOGITS_ALL
            shape = (B, 1 if logits == "last" else S, self.cfg.vocab_size)
        else:
            mode = _lib.MG_OUT_HIDDEN
            shape = (B, S, self.cfg.hidden_size)
        out = torch.empty(shape, dtype=self.dtype, device=self.device)
        _lib.check(
            self._lib.mg_stage_forward(
                self.handle,
                slot,
                _ptr(ids),
                None if self.has_embedding else _ptr(x),
                _ptr(pos),
                B,
                S,
                mode,
                out.data_ptr(),
                _stream(self.device),
            )
        )
        return out

    def decode_multi(
        self,
        slots: list[int],
        x: torch.Tensor | None,
        *,
        input_ids: torch.Tensor | None = None,
        logits: str = "last",
    ) -> torch.Tensor:
        """One single-token decode step for several slots in one weight pass.

        Rows are stacked in slot order: ``input_ids`` is [sum(B_slot), 1] on
        the first stage, ``x`` is [sum(B_slot), 1, H] elsewhere.
        """
        rows = sum(self.kv_batch(s) for s in slots)
        arr = (ctypes.c_int32 * len(slots))(*slots)
        ids = None
        if self.has_embedding:
            if input_ids is None or input_ids.shape[0] != rows:
                raise ValueError(f"decode_multi needs input_ids with {rows} rows")
            ids = input_ids.to(device=self.device, dtype=torch.int64).contiguous()
        else:
            if x is None or x.shape[0] != rows or x.shape[-1] != self.cfg.hidden_size:
                raise ValueError(f"decode_multi needs hidden states with {rows} rows")
            x = x.to(self.device).contiguous()
        if self.has_lm_head:
            mode = _lib.MG_OUT_LOGITS_LAST if logits == "last" else _lib.MG_OUT_LOGITS_ALL
            shape = (rows, 1, self.cfg.vocab_size)
        else:
            mode = _lib.MG_OUT_HIDDEN
            shape = (rows, 1, self.cfg.hidden_size)
        out = torch.empty(shape, dtype=self.dtype, device=self.device)
        _lib.check(
            self._lib.mg_stage_decode_multi(
                self.handle, arr, len(slots), _ptr(ids), None if self.has_embedding else _ptr(x),
                mode, out.data_ptr(), _stream(self.device),
            )
        )
        return out

    def decode_greedy(
        self,
        slots: list[int],
        x: torch.Tensor | None,
        *,
        input_ids: torch.Tensor | None = None,
        return_logits: bool = False,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        """``decode_multi`` on the last stage with each row's greedy token
        chosen on the device (fused into lm_head for the bf16 decode GEMM).

        Returns (token ids int64 [rows] on the stage's device, logits
        [rows, 1, V] or None).  The ids equal ``greedy_sample`` of the logits.
        """
        if not self.has_lm_head:
            raise ValueError("decode_greedy runs on the last stage")
        rows = sum(self.kv_batch(s) for s in slots)
        arr = (ctypes.c_int32 * len(slots))(*slots)
        ids = None
        if self.has_embedding:
            if input_ids is None or input_ids.shape[0] != rows:
                raise ValueError(f"decode_greedy needs input_ids with {rows} rows")
            ids = input_ids.to(device=self.device, dtype=torch.int64).contiguous()
        else:
            if x is None or x.shape[0] != rows or x.shape[-1] != self.cfg.hidden_size:
                raise ValueError(f"decode_greedy needs hidden states with {rows} rows")
            x = x.to(self.device).contiguous()
        tokens = torch.empty(rows, dtype=torch.int64, device=self.device)
        logits = (torch.empty((rows, 1, self.cfg.vocab_size), dtype=self.dtype, device=self.device)
                  if return_logits else None)
        _lib.check(
            self._lib.mg_stage_decode_greedy(
                self.handle, arr, len(slots), _ptr(ids), None if self.has_embedding else _ptr(x),
                tokens.data_ptr(), _ptr(logits), _stream(self.device),
            )
        )
        return tokens, logits

    def decode_top_p(
        self,
        slots: list[int],
        x: torch.Tensor | None,
        *,
        temperature: float,
        top_p: float,
        uniforms: torch.Tensor,
        input_ids: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """``decode_multi`` on the last stage with each row's top-p token drawn
        on the device for ``uniforms[r]`` (the selection counts the logits by
        value in the lm_head's epilogue).  Returns (token ids int64 [rows],
        logits [rows, 1, V])."""
        if not self.has_lm_head:
            raise ValueError("decode_top_p runs on the last stage")
        rows = sum(self.kv_batch(s) for s in slots)
        arr = (ctypes.c_int32 * len(slots))(*slots)
        ids = None
        if self.has_embedding:
            if input_ids is None or input_ids.shape[0] != rows:
                raise ValueError(f"decode_top_p needs input_ids with {rows} rows")
            ids = input_ids.to(device=self.device, dtype=torch.int64).contiguous()
        else:
            if x is None or x.shape[0] != rows or x.shape[-1] != self.cfg.hidden_size:
                raise ValueError(f"decode_top_p needs hidden states with {rows} rows")
            x = x.to(self.device).contiguous()
        u = uniforms.to(device=self.device, dtype=torch.float32).reshape(-1).contiguous()
        if u.numel() != rows:
            raise ValueError(f"decode_top_p needs one uniform per row ({rows})")
        tokens = torch.empty(rows, dtype=torch.int64, device=self.device)
        logits = torch.empty((rows, 1, self.cfg.vocab_size), dtype=self.dtype, device=self.device)
        _lib.check(
            self._lib.mg_stage_decode_top_p(
                self.handle, arr, len(slots), _ptr(ids), None if self.has_embedding else _ptr(x),
                float(temperature), float(top_p), u.data_ptr(), tokens.data_ptr(), logits.data_ptr(),
                _stream(self.device),
            )
        )
        return tokens, logits

    def profile(self, enable: bool) -> None:
        """Time every launch group with CUDA events (resets on enable)."""
        _lib.check(self._lib.mg_stage_profile(self.handle, int(enable)))

    def profile_read(self) -> dict[str, dict[str, float]]:
        prof = _lib.Profile()
        _lib.check(self._lib.mg_stage_profile_read(self.handle, ctypes.byref(prof)))
        return prof.as_dict()

    def probe_wait(self, limit_us: int, *, flag_set: bool = False) -> None:
        """Queue a bounded wait for the stage's probe flag (set only with
        ``flag_set``); unset, it runs out after ``limit_us`` and records the
        timeout code, which the next ``check_device`` raises as
        ``DeviceTimeoutError``."""
        _lib.check(self._lib.mg_stage_probe_wait(self.handle, int(limit_us), int(flag_set),
                                                 _stream(self.device)))

    def check_device(self) -> None:
        """Raise if a kernel clamped an out-of-range id or position since the last check."""
        _lib.check(self._lib.mg_stage_check_device(self.handle, _stream(self.device)))

    # ------------------------------------------------------------------
    # Parameters: views of the stage's HBM arena under the reference's names
    # ------------------------------------------------------------------
    def _weight_view(self, which: int, layer: int, shape: tuple[int, ...], row0: int = 0) -> torch.Tensor | None:
        ptr = ctypes.c_void_p()
        _lib.check(self._lib.mg_stage_weight(self.handle, which, layer, ctypes.byref(ptr)))
        if not ptr.value:
            return None
        esz = torch.empty((), dtype=self.dtype).element_size()
        typestr = {4: "<f4", 2: "<i2"}[esz]
        cols = shape[1] if len(shape) == 2 else 1
        arr = _DeviceArray(ptr.value + row0 * cols * esz, shape, typestr)
        t = torch.as_tensor(arr, device=self.device)
        return t if t.dtype == self.dtype else t.view(self.dtype)

    def named_parameters(self):
        """(reference name, tensor) for every weight, like LlamaStage's
        nn.Module parameters (llama_dense.py:293-348; Qwen3Stage adds q_norm /
        k_norm).  The tensors are views of the stage's own HBM copy: writing
        them changes the stage, and they are invalid after ``close()``."""
        cfg = self.cfg
        H, I, D, V = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim, cfg.vocab_size
        nq, nkv = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
        W = _lib
        if self.has_embedding:
            yield "embed_tokens.weight", self._weight_view(W.MG_W_EMBED, 0, (V, H))
        for i in range(self.layer_end - self.layer_start):
            p = f"layers.{i}."
            yield p + "self_attn.q_proj.weight", self._weight_view(W.MG_W_QKV, i, (nq, H))
            yield p + "self_attn.k_proj.weight", self._weight_view(W.MG_W_QKV, i, (nkv, H), nq)
            yield p + "self_attn.v_proj.weight", self._weight_view(W.MG_W_QKV, i, (nkv, H), nq + nkv)
            yield p + "self_attn.o_proj.weight", self._weight_view(W.MG_W_O, i, (H, nq))
            if cfg.qk_norm:
                yield p + "self_attn.q_norm.weight", self._weight_view(W.MG_W_Q_NORM, i, (D,))
                yield p + "self_attn.k_norm.weight", self._weight_view(W.MG_W_K_NORM, i, (D,))
            yield p + "mlp.gate_proj.weight", self._weight_view(W.MG_W_GATE_UP, i, (I, H))
            yield p + "mlp.up_proj.weight", self._weight_view(W.MG_W_GATE_UP, i, (I, H), I)
            yield p + "mlp.down_proj.weight", self._weight_view(W.MG_W_DOWN, i, (H, I))
            yield p + "input_layernorm.weight", self._weight_view(W.MG_W_INPUT_NORM, i, (H,))
            yield p + "post_attention_layernorm.weight", self._weight_view(W.MG_W_POST_NORM, i, (H,))
        if self.has_lm_head:
            yield "norm.weight", self._weight_view(W.MG_W_NORM, 0, (H,))
            head = self._weight_view(W.MG_W_LM_HEAD, 0, (V, H))
            embed = self._weight_view(W.MG_W_EMBED, 0, (V, H)) if self.has_embedding else None
            if embed is None or head.data_ptr() != embed.data_ptr():  # a tied head is listed once
                yield "lm_head.weight", head

    def parameters(self):
        for _, t in self.named_parameters():
            yield t

    # The reference stage's submodules, as weight views (absent where the
    # reference's would be: no embedding off the first stage, no head off the last).
    @property
    def embed_tokens(self) -> _Submodule:
        if not self.has_embedding:
            raise AttributeError("this stage has no embed_tokens")
        return _Submodule(self, "embed_tokens")

    @property
    def norm(self) -> _Submodule:
        if not self.has_lm_head:
            raise AttributeError("this stage has no norm")
        return _Submodule(self, "norm")

    @property
    def lm_head(self) -> _Submodule:
        if not self.has_lm_head:
            raise AttributeError("this stage has no lm_head")
        return _Submodule(self, "lm_head")

    @property
    def layers(self) -> list[_Submodule]:
        return [_Submodule(self, f"layers.{i}") for i in range(self.layer_end - self.layer_start)]

    def state_dict(self) -> dict[str, torch.Tensor]:
        """Every weight under its reference name (a tied head under both names)."""
        out = dict(self.named_parameters())
        if self.has_lm_head and "lm_head.weight" not in out:
            out["lm_head.weight"] = out["embed_tokens.weight"]
        return out

    def load_state_dict(self, state_dict: dict[str, torch.Tensor], strict: bool = True):
        """Copy weights into the stage (on its stream); torch's return value and
        ``strict`` semantics.  Buffers the reference does not persist (RoPE
        tables) are ignored."""
        own = self.state_dict()
        unexpected = [k for k in state_dict if k not in own and "rope" not in k and "rotary" not in k]
        missing = [k for k in own if k not in state_dict]
        if strict and (missing or unexpected):
            raise RuntimeError(f"Error(s) in loading state_dict for B200Stage: missing keys {missing}, "
                               f"unexpected keys {unexpected}")
        with torch.no_grad(), torch.cuda.device(self.device):
            for k, dst in own.items():
                if k in state_dict:
                    src = state_dict[k]
                    if tuple(src.shape) != tuple(dst.shape):
                        raise RuntimeError(f"size mismatch for {k}: copying a param with shape "
                                           f"{tuple(src.shape)}, the stage has {tuple(dst.shape)}")
                    dst.copy_(src.detach().to(device=self.device, dtype=self.dtype))
        return _LoadResult(missing, unexpected)

    # Reference-compatible cache helpers (Qwen3Stage.cache_length / trim_cache,
    # models/qwen3_hf.py:310-331), keyed by slot.
    def cache_length(self, slot: int) -> int:
        return self.kv_length(slot)

    def trim_cache(self, slot: int, length: int) -> None:
        self.kv_trim(slot, length)
