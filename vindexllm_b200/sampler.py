"""Host-side mirror of VindexLLM's sampler interface over the C ABI.

``TVdxSampler`` keeps the reference's method names and meaning (src/VindexLLM.Sampler.pas:
DefaultConfig :100-109, SetConfig :132-150, GetConfig :152-155, Process :265-528,
AddToHistory :530-539, ResetHistory :541-549) for a batch of rows, each with its own
PRNG and history ring. ``SamplerContext.sample`` is the stateless batched call
(vdxs_sample_ex). torch only supplies device memory and streams; all sampling runs in
libvdxsampler.so, and a missing library raises instead of falling back.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import abi
from ._lib import load, check, VdxsError
from .abi import VdxsConfig, default_config

__all__ = ["SamplerContext", "TVdxSampler", "ShardComm", "DeviceDecodeState", "VdxsError", "default_config",
           "shard_range", "broadcast_unique_id"]


def _stream_ptr(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(int(stream.cuda_stream))


def _dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return abi.DTYPE_F32
    if t.dtype == torch.bfloat16:
        return abi.DTYPE_BF16
    raise TypeError(f"logits must be float32 or bfloat16, got {t.dtype}")


def _dptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


class SamplerContext:
    """One vdxs_context: a device plus its lazily grown workspace."""

    def __init__(self, device: int = 0, tie_mode: int = abi.TIES_FAITHFUL):
        self.lib = load()
        h = C.c_void_p()
        check(self.lib.vdxs_create(device, C.byref(h)))
        self._h = h
        self.device = device
        self.set_tie_mode(tie_mode)

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            self.lib.vdxs_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tie_mode(self, mode: int):
        check(self.lib.vdxs_set_tie_mode(self._h, mode), self._h)

    def device_status(self, stream=None):
        """vdxs_device_status: waits for the stream, raises VdxsError if a kernel of an
        earlier call reported a timeout or a failed internal check."""
        check(self.lib.vdxs_device_status(self._h, _stream_ptr(stream)), self._h)

    def set_stage_events(self, ev_begin=None, ev_end=None):
        """Records two torch.cuda.Event objects around the dominant pass of every later
        call (None, None stops). The events are created here if torch has not yet."""
        if ev_begin is None or ev_end is None:
            check(self.lib.vdxs_set_stage_events(self._h, None, None), self._h)
            return
        for ev in (ev_begin, ev_end):
            if not ev.cuda_event:
                ev.record()
        check(self.lib.vdxs_set_stage_events(self._h, C.c_void_p(ev_begin.cuda_event),
                                             C.c_void_p(ev_end.cuda_event)), self._h)

    def launch_count(self) -> int:
        """Kernels the library has launched for this context."""
        n = C.c_int64()
        check(self.lib.vdxs_get_launch_count(self._h, C.byref(n)), self._h)
        return n.value

    def sample(self, cfg: VdxsConfig, logits, uniforms=None, history=None, history_count=None,
               vocab: int | None = None, out_k: int = 0, want_flags: bool = False, stream=None,
               tokens=None):
        """Stateless batched sampling on device tensors. Returns tokens, or
        (tokens, flags, idx, prob) when diagnostics are requested."""
        import torch
        assert logits.is_cuda and logits.dim() == 2 and logits.stride(1) == 1
        B, _ = logits.shape
        V = logits.shape[1] if vocab is None else vocab
        dev = logits.device
        if tokens is None:
            tokens = torch.empty(B, dtype=torch.int32, device=dev)
        flags = torch.empty(B, dtype=torch.int32, device=dev) if (want_flags or out_k) else None
        oi = torch.empty(B, out_k, dtype=torch.int32, device=dev) if out_k else None
        op = torch.empty(B, out_k, dtype=torch.float32, device=dev) if out_k else None
        hs = history.shape[1] if history is not None else 1
        rc = self.lib.vdxs_sample_ex(self._h, C.byref(cfg), _dptr(logits), _dtype_code(logits), B, V,
                                     logits.stride(0), _dptr(history), hs, _dptr(history_count),
                                     _dptr(uniforms), _dptr(tokens), _dptr(flags), _dptr(oi), _dptr(op),
                                     out_k, _stream_ptr(stream))
        check(rc, self._h)
        if flags is None:
            return tokens
        return tokens, flags, oi, op

    def sample_host(self, cfg: VdxsConfig, logits: np.ndarray, uniforms=None, history=None,
                    history_count=None, vocab: int | None = None, stream=None, out=None):
        """Host-buffer call (vdxs_sample_host): numpy (or pinned torch CPU) inputs, host tokens."""
        lg = logits
        if hasattr(lg, "numpy"):
            lg = lg.numpy()
        if lg.dtype == np.float32:
            dt = abi.DTYPE_F32
        elif lg.dtype in (np.uint16, np.int16):
            dt = abi.DTYPE_BF16
        else:
            raise TypeError("host logits must be float32 or bf16 bits (uint16)")
        B, S = lg.shape
        V = S if vocab is None else vocab
        out = np.empty(B, np.int32) if out is None else out

        def p(a):
            if a is None:
                return None
            if hasattr(a, "numpy"):
                a = a.numpy()
            return C.c_void_p(a.ctypes.data)
        hs = history.shape[1] if history is not None else 1
        rc = self.lib.vdxs_sample_host(self._h, C.byref(cfg), p(lg), dt, B, V, S, p(history), hs,
                                       p(history_count), p(uniforms), C.c_void_p(out.ctypes.data),
                                       _stream_ptr(stream) if stream is not None else None)
        check(rc, self._h)
        return out


class TVdxSampler:
    """TVdxSampler (Sampler.pas:37-91) for ``batch`` independent rows."""

    DefaultConfig = staticmethod(default_config)

    def __init__(self, ctx: SamplerContext, batch: int = 1):
        self.ctx = ctx
        self.lib = ctx.lib
        self.batch = batch
        h = C.c_void_p()
        check(self.lib.vdxs_sampler_create(ctx.handle, batch, C.byref(h)), ctx.handle)
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self.lib.vdxs_sampler_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def SetConfig(self, cfg: VdxsConfig):
        check(self.lib.vdxs_sampler_set_config(self._h, C.byref(cfg)), self.ctx.handle)

    def GetConfig(self) -> VdxsConfig:
        c = VdxsConfig()
        check(self.lib.vdxs_sampler_get_config(self._h, C.byref(c)), self.ctx.handle)
        return c

    def AddToHistory(self, token: int, row: int = 0):
        check(self.lib.vdxs_sampler_add_to_history(self._h, row, int(token)), self.ctx.handle)

    def AddToHistoryBatch(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(self.lib.vdxs_sampler_add_to_history_batch(self._h, C.c_void_p(t.ctypes.data)), self.ctx.handle)

    def ResetHistory(self, row: int = -1):
        check(self.lib.vdxs_sampler_reset_history(self._h, row), self.ctx.handle)

    def Process(self, logits, vocab: int | None = None, stream=None):
        """Process for every row. ``logits``: a CUDA tensor [batch, stride] (fp32/bf16), or a
        host float32 array [batch, stride] (the reference's PSingle calling shape).
        Returns an int32 numpy array of token ids (a Python int when batch == 1)."""
        out = np.empty(self.batch, np.int32)
        if isinstance(logits, np.ndarray):
            assert logits.dtype == np.float32 and logits.ndim in (1, 2)
            lg = np.ascontiguousarray(logits.reshape(self.batch, -1))
            V = lg.shape[1] if vocab is None else vocab
            check(self.lib.vdxs_sampler_process_host(self._h, C.c_void_p(lg.ctypes.data), V, lg.shape[1],
                                                     C.c_void_p(out.ctypes.data)), self.ctx.handle)
        else:
            lg = logits.reshape(self.batch, -1) if logits.dim() == 1 else logits
            V = lg.shape[1] if vocab is None else vocab
            check(self.lib.vdxs_sampler_process(self._h, _dptr(lg), _dtype_code(lg), V, lg.stride(0),
                                                C.c_void_p(out.ctypes.data), _stream_ptr(stream)),
                  self.ctx.handle)
        return int(out[0]) if self.batch == 1 else out

    def NextFloat(self, row: int = 0) -> float:
        f = C.c_float()
        check(self.lib.vdxs_sampler_next_float(self._h, row, C.byref(f)), self.ctx.handle)
        return f.value

    def GetPrngState(self, row: int = 0):
        st = (C.c_uint64 * 4)()
        check(self.lib.vdxs_sampler_get_prng_state(self._h, row, st), self.ctx.handle)
        return list(st)

    def SetPrngState(self, state, row: int = 0):
        check(self.lib.vdxs_sampler_set_prng_state(self._h, row, (C.c_uint64 * 4)(*state)), self.ctx.handle)

    def GetHistory(self, row: int = 0):
        cap = max(1, self.GetConfig().repeat_window)
        buf = (C.c_int32 * cap)()
        cnt, pos = C.c_int32(), C.c_int32()
        check(self.lib.vdxs_sampler_get_history(self._h, row, buf, cap, C.byref(cnt), C.byref(pos)),
              self.ctx.handle)
        return list(buf[: cnt.value]), cnt.value, pos.value


class DeviceDecodeState:
    """Row PRNGs and history rings kept on the device (vdxs_device_uniforms,
    vdxs_device_history_push, vdxs_decode_step), so a decode loop samples without a host
    round trip per token. The reference keeps both inside TVdxSampler on the host
    (Sampler.pas:157-248 PRNG, :530-549 ring); ``prng_states`` takes their 4-word states,
    e.g. from ``TVdxSampler.GetPrngState``."""

    def __init__(self, batch: int, window: int, device: int = 0, prng_states=None):
        import torch
        dev = torch.device("cuda", device)
        self.lib = load()
        self.batch, self.window = batch, window
        self.prng = torch.zeros((batch, 4), dtype=torch.int64, device=dev)  # uint64 bit patterns
        if prng_states is not None:
            st = np.ascontiguousarray(np.asarray(prng_states, dtype=np.uint64).reshape(batch, 4)).view(np.int64)
            self.prng.copy_(torch.from_numpy(st))
        self.uniforms = torch.zeros(batch, dtype=torch.float32, device=dev)
        self.hist = torch.zeros((batch, max(window, 1)), dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.count = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.stopped = torch.zeros(batch, dtype=torch.int32, device=dev)

    def next_uniforms(self, stream=None):
        """One NextFloat per row (Sampler.pas:243-248); returns the device tensor."""
        check(self.lib.vdxs_device_uniforms(_dptr(self.prng), self.batch, _dptr(self.uniforms), _stream_ptr(stream)))
        return self.uniforms

    def push(self, tokens, stop_ids=None, stream=None):
        """AddToHistory (Sampler.pas:530-539) of device tokens[batch]; flags stop tokens."""
        n_stop = 0 if stop_ids is None else int(stop_ids.numel())
        check(self.lib.vdxs_device_history_push(_dptr(self.hist), _dptr(self.pos), _dptr(self.count), self.window,
                                                _dptr(tokens), self.batch, _dptr(stop_ids), n_stop,
                                                _dptr(self.stopped), _stream_ptr(stream)))

    def step(self, ctx: "SamplerContext", cfg: VdxsConfig, logits, stop_ids=None, tokens=None, stream=None):
        """One device-resident decode step (vdxs_decode_step); returns the device tokens."""
        import torch
        assert logits.is_cuda and logits.dim() == 2 and logits.stride(1) == 1
        B, V = logits.shape
        assert B == self.batch and cfg.repeat_window == self.window
        if tokens is None:
            tokens = torch.empty(B, dtype=torch.int32, device=logits.device)
        n_stop = 0 if stop_ids is None else int(stop_ids.numel())
        check(self.lib.vdxs_decode_step(ctx._h, C.byref(cfg), _dptr(logits), _dtype_code(logits), B, V,
                                        logits.stride(0), _dptr(self.prng), _dptr(self.uniforms), _dptr(self.hist),
                                        _dptr(self.pos), _dptr(self.count), _dptr(stop_ids), n_stop,
                                        _dptr(self.stopped), _dptr(tokens), _stream_ptr(stream)), ctx._h)
        return tokens


def shard_range(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous vocab shard [lo, hi) of `rank`: the first vocab % world ranks hold one
    extra token, so every id has exactly one owner and shards are in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    q, r = divmod(vocab, world)
    lo = rank * q + min(rank, r)
    return lo, lo + q + (1 if rank < r else 0)


def broadcast_unique_id(rank: int, src: int = 0) -> bytes:
    """NCCL unique id made on `src` and shared through the caller's torch.distributed
    process group (any backend): what each rank passes to ShardComm."""
    import torch.distributed as dist
    obj = [ShardComm.unique_id() if rank == src else None]
    dist.broadcast_object_list(obj, src=src)
    return obj[0]


class ShardComm:
    """An NCCL communicator owned by the library (vdxs_comm)."""

    def __init__(self, ctx: SamplerContext, nranks: int, rank: int, unique_id: bytes, timeout_ms: int = 60000):
        """Creates the communicator (non-blocking NCCL init under `timeout_ms`: a rank that
        never joins raises VdxsError with VDXS_E_TIMEOUT instead of hanging)."""
        self.ctx = ctx
        self.lib = ctx.lib
        assert len(unique_id) == 128
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        h = C.c_void_p()
        check(self.lib.vdxs_comm_create_ex(ctx.handle, nranks, rank, buf, int(timeout_ms), C.byref(h)), ctx.handle)
        self._h = h
        self.nranks = nranks
        self.rank = rank

    @staticmethod
    def unique_id() -> bytes:
        lib = load()
        buf = (C.c_uint8 * 128)()
        check(lib.vdxs_comm_unique_id(buf))
        return bytes(buf)

    def close(self):
        if getattr(self, "_h", None):
            self.lib.vdxs_comm_destroy(self._h)
            self._h = None

    def abort(self):
        """vdxs_comm_abort: for a caller that learned on the host that a peer left."""
        check(self.lib.vdxs_comm_abort(self._h), self.ctx.handle)

    def status(self):
        """vdxs_comm_status: raises VdxsError after an asynchronous NCCL error or an abort."""
        check(self.lib.vdxs_comm_status(self._h), self.ctx.handle)

    def wait(self, stream=None, timeout_ms: int = 0):
        """vdxs_comm_wait: bounded wait for the stream; aborts the communicator on failure."""
        check(self.lib.vdxs_comm_wait(self._h, _stream_ptr(stream), int(timeout_ms)), self.ctx.handle)

    def sample(self, cfg: VdxsConfig, logits_shard, vocab_offset: int, vocab_total: int, uniforms=None,
               history=None, history_count=None, want_flags: bool = False, stream=None, tokens=None):
        import torch
        B, V = logits_shard.shape
        if tokens is None:
            tokens = torch.empty(B, dtype=torch.int32, device=logits_shard.device)
        flags = torch.empty(B, dtype=torch.int32, device=logits_shard.device) if want_flags else None
        hs = history.shape[1] if history is not None else 1
        rc = self.lib.vdxs_sample_sharded(self.ctx.handle, self._h, C.byref(cfg), _dptr(logits_shard),
                                          _dtype_code(logits_shard), B, V, logits_shard.stride(0),
                                          vocab_offset, vocab_total, _dptr(history), hs, _dptr(history_count),
                                          _dptr(uniforms), _dptr(tokens), _dptr(flags), _stream_ptr(stream))
        check(rc, self.ctx.handle)
        return (tokens, flags) if want_flags else tokens


class Q4Weights:
    """A Q4_0 unembedding matrix prepared on a context's device (vdxs_q4_0_prepare):
    TVdxModel.UnembedToLogits (src/VindexLLM.Model.pas:1258-1271) with the matvec of
    shaders/matvec_q4_0.comp, in front of the sampler."""

    def __init__(self, ctx: SamplerContext, q4_0, in_dim: int, out_dim: int, stream=None):
        """``q4_0``: a uint8 CUDA tensor holding [out_dim, in_dim / 32 * 18] Q4_0 blocks."""
        assert q4_0.is_cuda and q4_0.is_contiguous() and q4_0.numel() == out_dim * (in_dim // 32) * 18
        self.ctx = ctx
        self.lib = ctx.lib
        self.in_dim, self.out_dim = in_dim, out_dim
        h = C.c_void_p()
        check(self.lib.vdxs_q4_0_prepare(ctx.handle, _dptr(q4_0), in_dim, out_dim, _stream_ptr(stream),
                                         C.byref(h)), ctx.handle)
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self.lib.vdxs_q4_0_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def unembed(self, hidden, logits=None, stream=None):
        """logits [batch, out_dim] float32 = hidden [batch, in_dim] x weights^T."""
        import torch
        assert hidden.is_cuda and hidden.dtype == torch.float32 and hidden.is_contiguous()
        hidden = hidden.reshape(-1, self.in_dim)
        if logits is None:
            logits = torch.empty(hidden.shape[0], self.out_dim, dtype=torch.float32, device=hidden.device)
        check(self.lib.vdxs_unembed_q4_0(self.ctx.handle, self._h, _dptr(hidden), hidden.shape[0], _dptr(logits),
                                         _stream_ptr(stream)), self.ctx.handle)
        return logits

    def sample(self, cfg: VdxsConfig, hidden, uniforms=None, history=None, history_count=None, tokens=None,
               stream=None):
        """vdxs_sample_unembed_q4_0: unembedding and sampling in one call; returns tokens."""
        import torch
        assert hidden.is_cuda and hidden.dtype == torch.float32 and hidden.is_contiguous()
        hidden = hidden.reshape(-1, self.in_dim)
        B = hidden.shape[0]
        if tokens is None:
            tokens = torch.empty(B, dtype=torch.int32, device=hidden.device)
        hs = history.shape[1] if history is not None else 1
        check(self.lib.vdxs_sample_unembed_q4_0(self.ctx.handle, C.byref(cfg), self._h, _dptr(hidden), B,
                                                _dptr(history), hs, _dptr(history_count), _dptr(uniforms),
                                                _dptr(tokens), _stream_ptr(stream)), self.ctx.handle)
        return tokens
