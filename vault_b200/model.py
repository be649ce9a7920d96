"""Drop-in VAULT v3 streaming model on the B200 engine.

Mirrors the public inference API of the reference's src/vault_v3_model.py:
    VAULTv3ForCausalLM.new_state(batch, seg_budget)            :2159
    VAULTv3ForCausalLM.prefill(input_ids, vault_on, seg_budget)  :2163-2212  -> (logits [B, V], state)
    VAULTv3ForCausalLM.step(token_ids, st, vault_on)            :2214-2311  -> logits [B, V]
    VAULTv3ForCausalLM.forward(input_ids, mode, vault_on, seg_budget)  :2153  -> logits [B, L, V]
    VAULTv3State.pos / .n_pin / .set_pinned / .mem_pos / .nbytes       :974-1024
Weights come from a VLT3 file (tools/vlt3.py format) and stay quantized on the device.  Every computation runs in
the CUDA library through its C ABI; torch is used only to hold device buffers and to name the current stream.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Tuple, Union

import numpy as np
import torch

from . import _lib
from .config import VAULTv3Config
from .vlt3 import VLT3Error, aligned_buffer


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def sample_topk(logits: torch.Tensor, k: int, temp: float, rng: torch.Tensor) -> torch.Tensor:
    """Top-k (k <= 64) + temperature sampling of logit rows on the device: v3_sample_topk (runtime/vault3.c:3204-3230)
    per row.  logits: [B, V] fp32 on the GPU; rng: [B] int64 xorshift64 states on the same device (the reference's
    uint64 state as bits), updated in place; returns int32 tokens [B].  temp <= 0 or k <= 1: greedy."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_cuda or logits.stride(1) != 1:
        raise ValueError("logits must be a [B, V] fp32 CUDA tensor with contiguous rows")
    if rng.shape != (logits.shape[0],) or rng.dtype != torch.int64 or rng.device != logits.device or \
            not rng.is_contiguous():
        raise ValueError("rng must be a contiguous [B] int64 tensor on the logits' device")
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    with torch.cuda.device(logits.device):
        _lib.check(_lib.lib().v3g_sample_topk(C.c_void_p(logits.data_ptr()), logits.shape[0], logits.shape[1],
                                              logits.stride(0), int(k), float(temp), C.c_void_p(rng.data_ptr()),
                                              C.c_void_p(out.data_ptr()), _stream()), "v3g_sample_topk")
    return out


class Governor:
    """CAAI output governor (runtime/vault3.h:191-216): forbidden patterns built on the host, one stream state per
    sequence on the device.  govern() masks, in place, the candidate tokens that would complete a pattern
    (v3_govern_logits); commit() appends the chosen tokens to the streams (v3_gov_commit); pass the governor to
    VAULTv3ForCausalLM.generate to run both inside the on-device loop."""

    def __init__(self, batch: int = 1, device: Optional[Union[int, torch.device]] = None):
        self.rules = _lib.GovRules()
        _lib.lib().v3g_gov_init(C.byref(self.rules))
        dev = torch.device("cuda", device) if isinstance(device, int) else (device or torch.device("cuda"))
        self.streams = torch.zeros(batch, _lib.GOV_STREAM_BYTES, dtype=torch.uint8, device=dev)

    @property
    def active(self) -> bool:
        return self.rules.n_rules > 0

    def add_rule(self, pattern: bytes) -> None:
        _lib.check(_lib.lib().v3g_gov_add_rule(C.byref(self.rules), pattern, len(pattern)), "v3g_gov_add_rule")

    def arm_system(self, text: bytes) -> None:
        """Reset, then derive the rules from a system prompt (v3_gov_arm_system)."""
        _lib.lib().v3g_gov_arm_system(C.byref(self.rules), text, len(text))

    def reset_stream(self) -> None:
        self.streams.zero_()

    def govern(self, model: "VAULTv3ForCausalLM", logits: torch.Tensor, top_k_guard: int = 64) -> torch.Tensor:
        if logits.dim() != 2 or logits.dtype != torch.float32 or logits.stride(1) != 1 or \
                logits.shape[0] != self.streams.shape[0] or logits.shape[1] < model.cfg.vocab_size:
            raise ValueError("logits must be [batch, >= vocab] fp32 with contiguous rows")
        with torch.cuda.device(logits.device):
            _lib.check(_lib.lib().v3g_govern_logits(model._h, C.byref(self.rules), C.c_void_p(self.streams.data_ptr()),
                                                    C.c_void_p(logits.data_ptr()), logits.shape[0], logits.stride(0),
                                                    int(top_k_guard), _stream()), "v3g_govern_logits")
        return logits

    def commit(self, model: "VAULTv3ForCausalLM", tokens: torch.Tensor) -> None:
        tok = tokens.to(device=self.streams.device, dtype=torch.int32).reshape(-1).contiguous()
        if tok.numel() != self.streams.shape[0]:
            raise ValueError("one token per sequence")
        with torch.cuda.device(tok.device):
            _lib.check(_lib.lib().v3g_gov_commit(model._h, C.byref(self.rules), C.c_void_p(self.streams.data_ptr()),
                                                 C.c_void_p(tok.data_ptr()), tok.numel(), _stream()), "v3g_gov_commit")


class VAULTv3State:
    """Fixed-size streaming state held in a device arena (the reference's VAULTv3State / v3_state)."""

    def __init__(self, model: "VAULTv3ForCausalLM", batch: int = 1, seg_budget: Optional[int] = None,
                 per_sequence_memory: bool = False, auto_pin: bool = True, graphs: bool = True,
                 persistent: bool = True, chunked_prefill: bool = True, fp16_activations: bool = False):
        self.model = model
        self.batch = int(batch)
        cfg = model.cfg
        budget = cfg.seg_budget if seg_budget is None else int(seg_budget)
        if self.batch > 1 and not per_sequence_memory:
            budget = 0          # reference batched step: sliding window + sinks only (src/vault_v3_model.py:2194)
        self.seg_capacity = budget if cfg.seg_layers else 0
        L = _lib.lib()
        size = L.v3g_state_arena_size(model._h, self.batch, self.seg_capacity)
        if size == 0:
            raise ValueError("invalid state arguments")
        self.arena = torch.empty(int(size), dtype=torch.uint8, device=model.device)
        flags = (_lib.V3G_STATE_PER_SEQ_MEMORY if per_sequence_memory else 0) | \
                (0 if auto_pin else _lib.V3G_STATE_NO_AUTOPIN) | (0 if graphs else _lib.V3G_STATE_NO_GRAPHS) | \
                (0 if persistent else _lib.V3G_STATE_NO_PERSISTENT) | \
                (0 if chunked_prefill else _lib.V3G_STATE_TOKEN_PREFILL) | \
                (_lib.V3G_STATE_FP16_ACTIVATIONS if fp16_activations else 0)
        h = C.c_void_p()
        with torch.cuda.device(model.device):
            _lib.check(L.v3g_state_init(C.byref(h), model._h, C.c_void_p(self.arena.data_ptr()), int(size),
                                        self.batch, self.seg_capacity, flags), "v3g_state_init")
        self._h = h
        self.seg_budget = budget if cfg.seg_layers else 0
        if self.seg_budget > 0 and (self.batch == 1 or per_sequence_memory):
            _lib.check(L.v3g_set_seg_budget(h, self.seg_budget, _stream()), "v3g_set_seg_budget")
        self.seg_active = cfg.has_seg_scorer and self.seg_budget > 0 and (self.batch == 1 or per_sequence_memory)
        if self.batch > 1 and not per_sequence_memory:
            self.set_pinned(min(cfg.n_sink, cfg.window))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().v3g_state_free(h)
            except Exception:
                pass
            self._h = None

    @property
    def pos(self) -> int:
        return int(_lib.lib().v3g_state_pos(self._h))

    def info(self, b: int = 0, with_bank: bool = False):
        si = _lib.SeqInfo()
        cap = max(1, self.seg_capacity)
        mp = np.zeros(cap, np.int64)
        ms = np.zeros(cap, np.float32)
        _lib.check(_lib.lib().v3g_seq_info(self._h, b, C.byref(si), mp.ctypes.data_as(C.c_void_p),
                                           ms.ctypes.data_as(C.c_void_p), cap, _stream()), "v3g_seq_info")
        if with_bank:
            return si, mp[:si.mem_cnt].copy(), ms[:si.mem_cnt].copy()
        return si

    @property
    def n_pin(self) -> int:
        return int(self.info().n_pin)

    @property
    def mem_pos(self) -> torch.Tensor:
        return torch.from_numpy(self.info(with_bank=True)[1])

    @property
    def mem_score(self) -> torch.Tensor:
        return torch.from_numpy(self.info(with_bank=True)[2])

    def set_pinned(self, n_pin: int) -> None:
        """Pin the first n_pin tokens as sinks (src/vault_v3_model.py:1013, runtime/vault3.c:898-910)."""
        cap = min(self.model.cfg.window, self.model.cfg.sink_cap)
        _lib.check(_lib.lib().v3g_set_pinned(self._h, max(0, min(int(n_pin), cap)), _stream()), "v3g_set_pinned")

    def reset(self) -> None:
        _lib.check(_lib.lib().v3g_state_reset(self._h, _stream()), "v3g_state_reset")

    def status(self, clear: bool = False) -> int:
        bits = C.c_uint32()
        _lib.check(_lib.lib().v3g_status(self._h, C.byref(bits), int(clear), _stream()), "v3g_status")
        return int(bits.value)

    def check(self) -> None:
        """Synchronize the engine stream and raise if the device set a status bit."""
        self._raise_for(self.status())

    def _poll_status(self) -> None:
        """Raise for status bits of an earlier step whose asynchronous copy has landed; never waits."""
        ev = getattr(self, "_status_event", None)
        if ev is not None and ev.query():
            self._status_event = None
            self._raise_for(int(self._status_host[0]))

    def _queue_status_copy(self) -> None:
        """Enqueue a copy of the sticky status bits into pinned host memory (one copy in flight at a time)."""
        if getattr(self, "_status_event", None) is not None:
            return
        if getattr(self, "_status_host", None) is None:
            self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        _lib.check(_lib.lib().v3g_status_copy(self._h, C.c_void_p(self._status_host.data_ptr()), _stream()),
                   "v3g_status_copy")
        self._status_event = torch.cuda.Event()
        self._status_event.record()   # the current stream: the one _stream() hands the engine

    @staticmethod
    def _raise_for(bits: int) -> None:
        if bits & _lib.V3G_STATUS_RESONANCE:
            raise NotImplementedError("shingle-resonance bias would be active for this stream (a non-pinned "
                                      "<|im_end|> inside the last 38 tokens with > 2 bank segments); the engine "
                                      "does not run it")
        if bits:
            raise RuntimeError(f"device status bits {bits:#x}")

    def nbytes(self) -> int:
        return int(self.arena.numel())


class VAULTv3ForCausalLM:
    """VAULT v3 model served by the sm_100a engine."""

    def __init__(self, vlt3: Union[str, bytes], device: Optional[Union[int, torch.device]] = None,
                 verify_crc: bool = True, max_sink: int = 512):
        if not torch.cuda.is_available():
            raise RuntimeError("VAULT v3 B200 engine needs a CUDA device (there is no CPU fallback)")
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                           (device.index if isinstance(device, torch.device) else int(device)))
        self.device = dev
        buf = aligned_buffer(vlt3)
        L = _lib.lib()
        h = C.c_void_p()
        with torch.cuda.device(dev):
            _lib.check(L.v3g_load(C.byref(h), C.c_void_p(buf.ctypes.data), buf.size, int(verify_crc), dev.index,
                                  int(max_sink)), "v3g_load")
        self._h = h
        info = _lib.ModelInfo()
        _lib.check(L.v3g_model_get_info(h, C.byref(info)), "v3g_model_get_info")
        self.info = info
        nf = info.seg_n_feat
        self.cfg = VAULTv3Config(
            vocab_size=info.vocab_size, d_model=info.d_model, n_layers=info.n_layers, n_heads=info.n_heads,
            n_kv_heads=info.n_kv_heads, head_dim=info.head_dim, d_ff=info.d_ff, rms_eps=info.rms_eps,
            rope_theta=info.rope_theta, tie_embeddings=bool(info.flags & 1), window=info.window, n_sink=info.n_sink,
            max_sink=int(max_sink), im_start_id=info.im_start_id, im_end_id=info.im_end_id,
            seg_budget=info.seg_budget if nf else 0, seg_hidden=info.seg_hidden if nf else 256,
            seg_min=info.seg_min if nf else 16, seg_max=info.seg_max if nf else 48,
            seg_layers=tuple(info.seg_layers[:nf]) if nf else ())

    @classmethod
    def from_vlt3(cls, path: str, **kw) -> "VAULTv3ForCausalLM":
        return cls(path, **kw)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().v3g_free(h)
            except Exception:
                pass
            self._h = None

    # ---- streaming API
    def new_state(self, batch: int = 1, seg_budget: Optional[int] = None, **kw) -> VAULTv3State:
        return VAULTv3State(self, batch, seg_budget=seg_budget, **kw)

    def _ids(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(device=self.device, dtype=torch.int32).contiguous()

    @torch.no_grad()
    def step(self, token_ids: torch.Tensor, st: VAULTv3State, vault_on: bool = False) -> torch.Tensor:
        """token_ids [B] -> logits [B, V] (fp32, on the engine device).  The device status bits are checked
        without synchronizing: each step with segment memory enqueues a copy of them, and a later step (or
        st.check(), which synchronizes) raises once that copy shows a bit -- NotImplementedError when the
        shingle-resonance bias would have been active, RuntimeError otherwise."""
        _ = vault_on
        ids = self._ids(token_ids.reshape(-1))
        if ids.numel() != st.batch:
            raise ValueError(f"expected {st.batch} token ids, got {ids.numel()}")
        st._poll_status()
        out = torch.empty(st.batch, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().v3g_step(st._h, C.c_void_p(ids.data_ptr()), C.c_void_p(out.data_ptr()), None,
                                       _stream()), "v3g_step")
        if st.seg_active:
            st._queue_status_copy()
        return out

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, vault_on: bool = False,
                seg_budget: Optional[int] = None, **state_kw) -> Tuple[torch.Tensor, VAULTv3State]:
        """Prefill a prompt from position 0 (window-aligned pieces through the tensor-core GEMMs, or token by token
        with chunked_prefill=False); returns last-token logits [B, V] and the state."""
        _ = vault_on
        B, Lq = input_ids.shape
        st = self.new_state(B, seg_budget=seg_budget, **state_kw)
        ids = self._ids(input_ids)
        out = torch.empty(B, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().v3g_prefill(st._h, C.c_void_p(ids.data_ptr()), Lq, Lq, C.c_void_p(out.data_ptr()),
                                          None, _stream()), "v3g_prefill")
        st.check()
        return out, st

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, mode: str = "block", vault_on: bool = False,
                seg_budget: Optional[int] = None) -> torch.Tensor:
        """All-position logits [B, L, V].  mode='block' is the streaming path (identical to the reference's
        chunk-recurrent / block-sliding forward); mode='full' equals it for L <= 2W."""
        _ = vault_on
        B, Lq = input_ids.shape
        if mode == "full" and Lq > 2 * self.cfg.window:
            raise NotImplementedError("mode='full' beyond 2W tokens is plain dense attention, not the streaming path")
        st = self.new_state(B, seg_budget=seg_budget)
        ids = self._ids(input_ids)
        out = torch.empty(B, Lq, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        tmp = torch.empty(B, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        L = _lib.lib()
        for t in range(Lq):
            col = ids[:, t].contiguous()
            _lib.check(L.v3g_step(st._h, C.c_void_p(col.data_ptr()), C.c_void_p(tmp.data_ptr()), None, _stream()),
                       "v3g_step")
            out[:, t] = tmp
        st.check()
        return out

    __call__ = forward

    @torch.no_grad()
    def generate(self, st: VAULTv3State, first_tokens: torch.Tensor, n_steps: int, top_k: int = 1,
                 temperature: float = 0.0, rng: Optional[torch.Tensor] = None,
                 governor: Optional[Governor] = None) -> torch.Tensor:
        """Decode n_steps tokens on the device starting from first_tokens [B]; returns int32 [B, n_steps].
        Greedy by default; with temperature > 0 and top_k > 1 every token is drawn by sample_topk's rule (the
        reference's v3_sample_topk) from the per-sequence xorshift states rng ([B] int64, advanced in place).
        With an armed governor each step's logits are masked and each token committed, as in
        runtime/vault3_host.c:586-606."""
        first = self._ids(first_tokens.reshape(-1))
        out = torch.empty(st.batch, n_steps, dtype=torch.int32, device=self.device)
        governed = governor is not None and governor.active
        if governed and governor.streams.shape[0] != st.batch:
            raise ValueError("the governor holds a stream per sequence: batch sizes differ")
        if (temperature > 0.0 and top_k > 1) or governed:
            if rng is None:
                rng = torch.zeros(st.batch, dtype=torch.int64, device=out.device)
            if rng.shape != (st.batch,) or rng.dtype != torch.int64 or rng.device != out.device or \
                    not rng.is_contiguous():
                raise ValueError("sampled generation needs rng: a contiguous [B] int64 tensor on the model's device")
            _lib.check(_lib.lib().v3g_generate_sampled(
                st._h, C.c_void_p(first.data_ptr()), n_steps, C.c_void_p(out.data_ptr()), n_steps, int(top_k),
                float(temperature), C.c_void_p(rng.data_ptr()), C.byref(governor.rules) if governed else None,
                C.c_void_p(governor.streams.data_ptr()) if governed else None, _stream()), "v3g_generate_sampled")
        else:
            _lib.check(_lib.lib().v3g_generate(st._h, C.c_void_p(first.data_ptr()), n_steps,
                                               C.c_void_p(out.data_ptr()), n_steps, _stream()), "v3g_generate")
        if st.seg_active:
            st.check()
        return out

    # ---- kernel-level access (tests, kernel sweep)
    def dequant(self, tensor_id: int, rows: int, cols: int) -> torch.Tensor:
        out = torch.empty(rows, cols, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().v3g_dequant(self._h, tensor_id, C.c_void_p(out.data_ptr()), _stream()), "v3g_dequant")
        return out

    def gemm(self, tensor_id: int, x: torch.Tensor, rows: int) -> torch.Tensor:
        """y [n_tok, rows] = x [n_tok, K] @ W^T on the tensor-core GEMM (the prefill / batched-decode kernel)."""
        x = x.to(device=self.device, dtype=torch.float32).contiguous()
        L = _lib.lib()
        n = x.shape[0]
        nbytes = int(L.v3g_gemm_work_size(self._h, tensor_id, n))
        work = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        y = torch.empty(n, rows, dtype=torch.float32, device=self.device)
        _lib.check(L.v3g_gemm(self._h, tensor_id, C.c_void_p(x.data_ptr()), n, C.c_void_p(y.data_ptr()),
                              C.c_void_p(work.data_ptr()), nbytes, _stream()), "v3g_gemm")
        return y

    def gemv(self, tensor_id: int, x: torch.Tensor, rows: int) -> torch.Tensor:
        x = x.to(device=self.device, dtype=torch.float32).contiguous()
        B = x.shape[0]
        y = torch.empty(B, rows, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().v3g_gemv(self._h, tensor_id, C.c_void_p(x.data_ptr()), B, C.c_void_p(y.data_ptr()),
                                       _stream()), "v3g_gemv")
        return y


__all__ = ["VAULTv3ForCausalLM", "VAULTv3State", "VAULTv3Config", "VLT3Error"]
