"""noetic_b200 -- the noetic language model's token loop on B200 GPUs.

Python mirror of the reference crate's inference API over the C ABI of
``libnoetic_gpu.so`` (declared in ``include/noetic_gpu.h``):

=====================================  ===========================================
reference (noetic crate)               here
=====================================  ===========================================
``LmConfig`` (model.rs:20-99)          :class:`LmConfig`
``Lm::new`` + ``Graph`` params         :class:`Model` (``Model.new(cfg, seed)``)
``ckpt::load`` + ``apply_exact``       :meth:`Model.load`
``Decoder`` (infer.rs:80-104)          :class:`Decoder` over ``n_streams`` streams
``SampleCfg`` (infer.rs:211-225)       :class:`SampleCfg`
``sample_token`` (infer.rs:228-305)    :func:`sample_token`, :meth:`Decoder.sample`
``cli.rs:generate`` (cli.rs:470-518)   :meth:`Decoder.generate`
``scan_sequential`` / ``scan_chunked`` :func:`scan_sequential`, :func:`scan_chunked`
``scan_adjoint`` (scan.rs:235-260)     :func:`scan_adjoint`
``gemm_tn`` (tensor.rs:156-198)        :func:`gemm_tn`
``Op::DwConv`` backward                :func:`dwconv_backward`
``AdamW::step`` (optim.rs:33-72)       :func:`adamw_step`
``Lm::loss`` (model.rs:228-234)        :meth:`Model.loss`
=====================================  ===========================================

Every computation runs on the GPU through hand-written sm_100a kernels.  There
is no CPU fallback: importing works without a GPU, but every call that needs
the library raises :class:`NoeticError` when the extension or a device is
missing.  Errors the reference reports with ``panic!`` / ``io::Error`` raise
:class:`NoeticError` with the library's status code and message.
"""

from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnoetic_gpu.so")

NK_OK, NK_ERR_INVALID, NK_ERR_CUDA, NK_ERR_OOM, NK_ERR_IO, NK_ERR_UNSUPPORTED, NK_ERR_DEVICE = range(7)

# Every entry point of include/noetic_gpu.h: name -> (restype, argtypes).
_P = C.c_void_p
_u32, _u64, _i32, _f32 = C.c_uint32, C.c_uint64, C.c_int, C.c_float


class NkConfig(C.Structure):
    _fields_ = [("vocab", _u64), ("d_model", _u64), ("n_layer", _u64), ("expand", _u64),
                ("conv_k", _u64), ("mlp_mult", _u64), ("eps", _f32), ("tau_max", _f32)]


class NkSampleCfg(C.Structure):
    _fields_ = [("temperature", _f32), ("top_k", _u64), ("top_p", _f32), ("rep_penalty", _f32),
                ("rep_window", _u64), ("greedy", _u32)]


class NkAdamwCfg(C.Structure):
    _fields_ = [("lr", _f32), ("b1", _f32), ("b2", _f32), ("eps", _f32), ("wd", _f32), ("t", _u64),
                ("decay", _i32)]


class NkProfile(C.Structure):
    _fields_ = [("proj_ms", C.c_double), ("proj_launches", _u64), ("proj_flops", C.c_double),
                ("proj_bytes", C.c_double), ("launches", _u64), ("tensor_core", _i32), ("sample_ms", C.c_double),
                ("sample_launches", _u64)]


SIGNATURES = {
    "nk_last_error": (C.c_char_p, []),
    "nk_device_count": (_i32, [C.POINTER(_i32)]),
    "nk_config_check": (_i32, [C.POINTER(NkConfig)]),
    "nk_model_create": (_i32, [C.POINTER(NkConfig), _i32, C.POINTER(_P)]),
    "nk_model_destroy": (_i32, [_P]),
    "nk_model_config": (_i32, [_P, C.POINTER(NkConfig)]),
    "nk_model_init_random": (_i32, [_P, _u64, _P]),
    "nk_model_tensor_count": (_i32, [_P, C.POINTER(_u64)]),
    "nk_model_tensor_info": (_i32, [_P, _u64, C.POINTER(C.c_char_p), C.POINTER(_u32), _P]),
    "nk_model_set_tensor": (_i32, [_P, C.c_char_p, _P, _P, _u32]),
    "nk_model_get_tensor": (_i32, [_P, C.c_char_p, _P, _u64]),
    "nk_model_load_ckpt": (_i32, [C.c_char_p, _i32, C.POINTER(_P)]),
    "nk_crc32": (_i32, [_P, _u64, C.POINTER(_u32)]),
    "nk_model_save_ckpt": (_i32, [_P, C.c_char_p]),
    "nk_model_loss": (_i32, [_P, _P, _P, _u32, _u32, C.POINTER(C.c_float), _P]),
    "nk_decoder_create": (_i32, [_P, _u32, C.POINTER(_P)]),
    "nk_decoder_destroy": (_i32, [_P]),
    "nk_decoder_streams": (_i32, [_P, C.POINTER(_u32)]),
    "nk_decoder_reset": (_i32, [_P, _u32, _u32]),
    "nk_decoder_step": (_i32, [_P, _P, _P]),
    "nk_decoder_prefill": (_i32, [_P, _P, _P, _u32, _P]),
    "nk_decoder_sample": (_i32, [_P, C.POINTER(NkSampleCfg), _P, _P, _u32, _P, _P]),
    "nk_decoder_generate": (_i32, [_P, _P, _P, _u32, _u32, C.POINTER(NkSampleCfg), _P, _P]),
    "nk_decoder_get_state": (_i32, [_P, _u32, _u32, _P, _P]),
    "nk_decoder_set_state": (_i32, [_P, _u32, _u32, _P, _P]),
    "nk_decoder_step_greedy_device": (_i32, [_P, _P, _P]),
    "nk_decoder_step_greedy": (_i32, [_P, _P, _P]),
    "nk_decoder_cuda_stream": (_i32, [_P, C.POINTER(_P)]),
    "nk_decoder_sync": (_i32, [_P]),
    "nk_decoder_set_engine": (_i32, [_P, _i32]),
    "nk_decoder_launch_count": (_i32, [_P, C.POINTER(_u64)]),
    "nk_decoder_profile_begin": (_i32, [_P]),
    "nk_decoder_profile_end": (_i32, [_P, C.POINTER(NkProfile)]),
    "nk_scan": (_i32, [_P, _P, _P, _u64, _u64, _u64, _i32, _i32]),
    "nk_scan_device": (_i32, [_P, _P, _P, _u64, _u64, _u64, _i32, _P]),
    "nk_scan_adjoint": (_i32, [_P, _P, _P, _u64, _u64, _u64, _i32, _i32]),
    "nk_bpe_create_bytes_only": (_i32, [C.POINTER(_P)]),
    "nk_bpe_load": (_i32, [C.c_char_p, C.POINTER(_P)]),
    "nk_bpe_save": (_i32, [_P, C.c_char_p]),
    "nk_bpe_destroy": (_i32, [_P]),
    "nk_bpe_vocab_size": (_i32, [_P, C.POINTER(_u64)]),
    "nk_bpe_merge": (_i32, [_P, _u64, C.POINTER(_u32), C.POINTER(_u32)]),
    "nk_bpe_encode": (_i32, [_P, _P, _u64, _P, _u64, C.POINTER(_u64)]),
    "nk_bpe_encode_bytes": (_i32, [_P, _P, _u64, _P, _u64, C.POINTER(_u64)]),
    "nk_bpe_decode_bytes": (_i32, [_P, _P, _u64, _P, _u64, C.POINTER(_u64)]),
    "nk_gemm_tn": (_i32, [_P, _P, _P, _u64, _u64, _u64, _i32]),
    "nk_gemm_tn_device": (_i32, [_P, _P, _P, _u64, _u64, _u64, _P]),
    "nk_dwconv_backward": (_i32, [_P, _P, _P, _P, _P, _P, _u64, _u64, _u64, _u64, _i32]),
    "nk_dwconv_backward_device": (_i32, [_P, _P, _P, _P, _P, _P, _u64, _u64, _u64, _u64, _P]),
    "nk_adamw_step": (_i32, [_P, _P, _P, _P, _u64, C.POINTER(NkAdamwCfg), _i32]),
    "nk_adamw_step_device": (_i32, [_P, _P, _P, _P, _u64, C.POINTER(NkAdamwCfg), _P]),
    "nk_scan_adjoint_device": (_i32, [_P, _P, _P, _u64, _u64, _u64, _i32, _P]),
    "nk_scan_chunked_noalloc_device": (_i32, [_P, _P, _P, _u64, _u64, _u64, _P]),
    "nk_sample_token": (_i32, [_P, _u64, C.POINTER(NkSampleCfg), _P, _u64, _P, _P, _i32]),
}

_lib = None


class NoeticError(RuntimeError):
    """A failing library call: ``.status`` is the nk_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[nk_status {status}] {message}")
        self.status = status


def lib():
    """Load ``libnoetic_gpu.so`` (raises :class:`NoeticError` if it is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NoeticError(NK_ERR_UNSUPPORTED,
                              f"{LIB_PATH} is not built; run python noetic_b200/make_lib.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(status: int):
    if status != NK_OK:
        raise NoeticError(status, lib().nk_last_error().decode(errors="replace"))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _u32a(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.uint32))


def device_count() -> int:
    n = C.c_int(0)
    _check(lib().nk_device_count(C.byref(n)))
    return n.value


# ---------------------------------------------------------------- configs
@dataclass
class LmConfig:
    """model.rs:20-30.  ``expand`` = E/d, ``mlp_mult`` = H/d."""

    vocab: int
    d_model: int = 128
    n_layer: int = 2
    expand: int = 2
    conv_k: int = 4
    mlp_mult: int = 3
    eps: float = 1e-5
    tau_max: float = 128.0

    @staticmethod
    def small(vocab: int) -> "LmConfig":  # model.rs:33-35
        return LmConfig(vocab, 128, 2, 2, 4, 3, 1e-5, 128.0)

    def c(self) -> NkConfig:
        return NkConfig(self.vocab, self.d_model, self.n_layer, self.expand, self.conv_k,
                        self.mlp_mult, self.eps, self.tau_max)

    def check(self):
        """LmConfig::check (model.rs:37-76); raises NoeticError."""
        _check(lib().nk_config_check(C.byref(self.c())))

    def inner(self) -> int:
        return self.d_model * self.expand

    def hidden(self) -> int:
        return self.d_model * self.mlp_mult

    def recurrent_projection(self) -> int:
        return 3 * self.inner()

    def mlp_projection(self) -> int:
        return 2 * self.hidden()


@dataclass
class SampleCfg:
    """infer.rs:211-225; ``SampleCfg.default_cfg()`` is the reference default."""

    temperature: float = 0.9
    top_k: int = 40
    top_p: float = 0.95
    rep_penalty: float = 1.1
    rep_window: int = 64
    greedy: bool = False

    @staticmethod
    def default_cfg() -> "SampleCfg":
        return SampleCfg()

    def c(self) -> NkSampleCfg:
        return NkSampleCfg(self.temperature, self.top_k, self.top_p, self.rep_penalty,
                           self.rep_window, 1 if self.greedy else 0)


def rng_state(seed: int) -> np.ndarray:
    """Rng::new(seed).s (rng.rs:25-38) as 4 x u64 -- the per-stream sampler state."""
    mask = (1 << 64) - 1
    z = (seed ^ 0xA0761D6478BD642F) & mask
    out = []
    for _ in range(4):
        z = (z + 0x9E3779B97F4A7C15) & mask
        r = z
        r = ((r ^ (r >> 30)) * 0xBF58476D1CE4E5B9) & mask
        r = ((r ^ (r >> 27)) * 0x94D049BB133111EB) & mask
        out.append(r ^ (r >> 31))
    if not any(out):
        out[0] = 0x9E3779B97F4A7C15
    return np.array(out, dtype=np.uint64)


# ---------------------------------------------------------------- model
class Model:
    """The model's parameters on one GPU (``Graph`` + ``Lm``, model.rs:175-206)."""

    def __init__(self, cfg: LmConfig, device: int = 0, _handle=None):
        self.cfg = cfg
        self.device = device
        if _handle is not None:
            self.h = _handle
        else:
            h = C.c_void_p()
            _check(lib().nk_model_create(C.byref(cfg.c()), device, C.byref(h)))
            self.h = h
        self.rng_after_init = None

    @classmethod
    def new(cls, cfg: LmConfig, seed: int, device: int = 0) -> "Model":
        """Lm::new(g, &mut Rng::new(seed), cfg): the reference's seeded init."""
        m = cls(cfg, device)
        after = np.zeros(4, dtype=np.uint64)
        _check(lib().nk_model_init_random(m.h, seed, _ptr(after)))
        m.rng_after_init = after
        return m

    @classmethod
    def load(cls, path: str, device: int = 0) -> "Model":
        """ckpt::load + apply_exact (ckpt.rs:299-436) into a new model."""
        h = C.c_void_p()
        _check(lib().nk_model_load_ckpt(os.fsencode(path), device, C.byref(h)))
        c = NkConfig()
        _check(lib().nk_model_config(h, C.byref(c)))
        cfg = LmConfig(c.vocab, c.d_model, c.n_layer, c.expand, c.conv_k, c.mlp_mult, c.eps, c.tau_max)
        return cls(cfg, device, _handle=h)

    def save(self, path: str):
        _check(lib().nk_model_save_ckpt(self.h, os.fsencode(path)))

    def loss(self, ids, targets, batch: int, t: int, want_logits: bool = False):
        """Lm::loss (model.rs:228-234): mean cross-entropy in nats of `batch`
        sequences of `t` tokens (targets 0xFFFFFFFF ignored); returns the loss,
        or (loss, logits [batch * t, vocab]) with want_logits."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
        targets = np.ascontiguousarray(targets, dtype=np.uint32).reshape(-1)
        if ids.size != batch * t or targets.size != batch * t:
            raise ValueError("ids and targets must hold batch * t entries")
        out = np.empty((batch * t, self.cfg.vocab), dtype=np.float32) if want_logits else None
        loss = C.c_float()
        _check(lib().nk_model_loss(self.h, _ptr(ids), _ptr(targets), batch, t, C.byref(loss),
                                   _ptr(out) if out is not None else None))
        return (float(loss.value), out) if want_logits else float(loss.value)

    def close(self):
        if getattr(self, "h", None):
            lib().nk_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor_names(self):
        n = C.c_uint64()
        _check(lib().nk_model_tensor_count(self.h, C.byref(n)))
        out = []
        for i in range(n.value):
            name = C.c_char_p()
            rank = C.c_uint32()
            shape = (C.c_uint64 * 4)()
            _check(lib().nk_model_tensor_info(self.h, i, C.byref(name), C.byref(rank), shape))
            out.append((name.value.decode(), tuple(int(shape[a]) for a in range(rank.value))))
        return out

    def set_tensor(self, name: str, data: np.ndarray):
        a = np.ascontiguousarray(data, dtype=np.float32)
        shape = np.asarray(a.shape, dtype=np.uint64)
        _check(lib().nk_model_set_tensor(self.h, name.encode(), _ptr(a), _ptr(shape), a.ndim))

    def get_tensor(self, name: str) -> np.ndarray:
        shape = dict(self.tensor_names())[name]
        out = np.empty(shape, dtype=np.float32)
        _check(lib().nk_model_get_tensor(self.h, name.encode(), _ptr(out), out.size))
        return out


# ---------------------------------------------------------------- decoder
class Decoder:
    """``Decoder`` (infer.rs:80-104) for ``n_streams`` independent streams."""

    def __init__(self, model: Model, n_streams: int = 1):
        self.model = model
        self.n_streams = n_streams
        h = C.c_void_p()
        _check(lib().nk_decoder_create(model.h, n_streams, C.byref(h)))
        self.h = h
        V = model.cfg.vocab
        self._logits = np.zeros((n_streams, V), dtype=np.float32)

    def close(self):
        if getattr(self, "h", None):
            lib().nk_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_engine(self, engine: int):
        """0 = automatic; bit 0 = f32 CUDA-core projections only; bit 1 / bit 2
        force the time-chunked / sequential prefill scan; bit 3 no fused
        few-stream step; bit 10 no persistent step kernel (1-4 streams take
        the fused small-batch kernels).  The C header lists every bit."""
        _check(lib().nk_decoder_set_engine(self.h, engine))

    def reset(self, first: int = 0, count: int | None = None):
        """LmState::reset (infer.rs:37-44) for streams [first, first+count)."""
        count = self.n_streams - first if count is None else count
        _check(lib().nk_decoder_reset(self.h, first, count))

    def step(self, tokens) -> np.ndarray:
        """Decoder::step for every stream; returns logits [S, vocab]."""
        t = _u32a(tokens).reshape(-1)
        if t.size != self.n_streams:
            raise NoeticError(NK_ERR_INVALID, "one token per stream is required")
        _check(lib().nk_decoder_step(self.h, _ptr(t), _ptr(self._logits)))
        return self._logits

    def logits_mut(self) -> np.ndarray:
        return self._logits

    def step_greedy(self, tokens) -> np.ndarray:
        t = _u32a(tokens).reshape(-1)
        out = np.empty(self.n_streams, dtype=np.uint32)
        _check(lib().nk_decoder_step_greedy(self.h, _ptr(t), _ptr(out)))
        return out

    def step_greedy_device(self, tokens_in_ptr: int, tokens_out_ptr: int):
        """Device-resident greedy step on u32[S] device buffers (asynchronous)."""
        _check(lib().nk_decoder_step_greedy_device(self.h, C.c_void_p(tokens_in_ptr),
                                                   C.c_void_p(tokens_out_ptr)))

    def prefill(self, ids, lens=None, want_logits: bool = True) -> np.ndarray | None:
        """Scan prefill of [S, T] prompts (ragged via ``lens``); returns the
        logits after each stream's last prompt token."""
        ids = _u32a(ids)
        if ids.ndim == 1:
            ids = ids.reshape(self.n_streams, -1)
        S, T = ids.shape
        lens = np.full(S, T, dtype=np.uint32) if lens is None else _u32a(lens)
        out = self._logits if want_logits else None
        _check(lib().nk_decoder_prefill(self.h, _ptr(ids), _ptr(lens), T,
                                        _ptr(out) if out is not None else None))
        return out

    def sample(self, cfg: SampleCfg, rng: np.ndarray, history=None, history_len=None) -> np.ndarray:
        """sample_token on every stream's current logits; ``rng`` [S,4] u64 is updated."""
        assert rng.dtype == np.uint64 and rng.shape == (self.n_streams, 4) and rng.flags["C_CONTIGUOUS"]
        out = np.empty(self.n_streams, dtype=np.uint32)
        if history is not None:
            hist = _u32a(history)
            hl = _u32a(history_len)
            _check(lib().nk_decoder_sample(self.h, C.byref(cfg.c()), _ptr(hist), _ptr(hl),
                                           hist.shape[1], _ptr(rng), _ptr(out)))
        else:
            _check(lib().nk_decoder_sample(self.h, C.byref(cfg.c()), None, None, 0, _ptr(rng), _ptr(out)))
        return out

    def generate(self, ids, lens, n_new: int, cfg: SampleCfg, rng: np.ndarray) -> np.ndarray:
        """cli.rs:generate for every stream; returns tokens [S, n_new]."""
        ids = _u32a(ids)
        if ids.ndim == 1:
            ids = ids.reshape(self.n_streams, -1)
        S, T = ids.shape
        lens = _u32a(lens)
        assert rng.dtype == np.uint64 and rng.shape == (S, 4) and rng.flags["C_CONTIGUOUS"]
        out = np.zeros((S, n_new), dtype=np.uint32)
        _check(lib().nk_decoder_generate(self.h, _ptr(ids), _ptr(lens), T, n_new, C.byref(cfg.c()),
                                         _ptr(rng), _ptr(out)))
        return out

    def get_state(self, first: int = 0, count: int | None = None):
        """State [count, n_layer, (k+1)*E] and heads [count]."""
        count = self.n_streams - first if count is None else count
        c = self.model.cfg
        st = np.empty((count, c.n_layer, (c.conv_k + 1) * c.inner()), dtype=np.float32)
        heads = np.empty(count, dtype=np.uint32)
        _check(lib().nk_decoder_get_state(self.h, first, count, _ptr(st), _ptr(heads)))
        return st, heads

    def set_state(self, state: np.ndarray, heads, first: int = 0):
        st = np.ascontiguousarray(state, dtype=np.float32)
        hd = _u32a(heads)
        _check(lib().nk_decoder_set_state(self.h, first, hd.size, _ptr(st), _ptr(hd)))

    def cuda_stream(self) -> int:
        p = C.c_void_p()
        _check(lib().nk_decoder_cuda_stream(self.h, C.byref(p)))
        return p.value or 0

    def sync(self):
        _check(lib().nk_decoder_sync(self.h))

    def launch_count(self) -> int:
        n = C.c_uint64()
        _check(lib().nk_decoder_launch_count(self.h, C.byref(n)))
        return n.value

    def profile_begin(self):
        _check(lib().nk_decoder_profile_begin(self.h))

    def profile_end(self) -> dict:
        p = NkProfile()
        _check(lib().nk_decoder_profile_end(self.h, C.byref(p)))
        return {"proj_ms": p.proj_ms, "proj_launches": p.proj_launches, "proj_flops": p.proj_flops,
                "proj_bytes": p.proj_bytes, "launches": p.launches, "tensor_core": bool(p.tensor_core),
                "sample_ms": p.sample_ms, "sample_launches": p.sample_launches}


# ---------------------------------------------------------------- ops
def _scan(a, b, batch, t, d, chunked, device):
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    if a.size != batch * t * d or b.size != batch * t * d:
        raise NoeticError(NK_ERR_INVALID, "scan: bad a/b")
    h = np.empty(batch * t * d, dtype=np.float32)
    _check(lib().nk_scan(_ptr(a), _ptr(b), _ptr(h), batch, t, d, 1 if chunked else 0, device))
    return h


def scan_sequential(a, b, batch: int, t: int, d: int, device: int = 0) -> np.ndarray:
    """scan.rs:35-57 on the GPU; returns h (flat, layout (b*T + t)*D + j)."""
    return _scan(a, b, batch, t, d, False, device)


def scan_chunked(a, b, batch: int, t: int, d: int, device: int = 0) -> np.ndarray:
    """scan.rs:98-225 (time-chunked associative scan) on the GPU."""
    return _scan(a, b, batch, t, d, True, device)


def scan_adjoint(a, g, batch: int, t: int, d: int, chunked: bool = False, device: int = 0) -> np.ndarray:
    """scan.rs:227-260 on the GPU: c_t = g_t + a_{t+1} c_{t+1}, c_T = 0; returns c
    (flat, layout (b*T + t)*D + j); chunked selects the time-parallel form."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    g = np.ascontiguousarray(g, dtype=np.float32).reshape(-1)
    n = batch * t * d
    if a.size != n or g.size != n:
        raise ValueError("a and g must hold batch * t * d values")
    c = np.empty(n, dtype=np.float32)
    _check(lib().nk_scan_adjoint(_ptr(a), _ptr(g), _ptr(c), batch, t, d, int(chunked), device))
    return c


class Bpe:
    """Byte-level BPE (bpe.rs) over ``nk_bpe_*``: tokens 0..255 are bytes,
    merge i makes token 256 + i.  Host only (no device needed)."""

    def __init__(self, handle):
        self.h = handle

    @staticmethod
    def bytes_only() -> "Bpe":
        """Bpe::bytes_only (bpe.rs:47-53)."""
        h = _P()
        _check(lib().nk_bpe_create_bytes_only(C.byref(h)))
        return Bpe(h)

    @staticmethod
    def load(path: str) -> "Bpe":
        """Bpe::load (bpe.rs:309-380); a bad file raises NoeticError (NK_ERR_IO)."""
        h = _P()
        _check(lib().nk_bpe_load(os.fsencode(path), C.byref(h)))
        return Bpe(h)

    def save(self, path: str):
        """Bpe::save (bpe.rs:288-307)."""
        _check(lib().nk_bpe_save(self.h, os.fsencode(path)))

    def vocab_size(self) -> int:
        n = _u64(0)
        _check(lib().nk_bpe_vocab_size(self.h, C.byref(n)))
        return n.value

    def merges(self) -> list:
        out = []
        for i in range(self.vocab_size() - 256):
            a, b = _u32(0), _u32(0)
            _check(lib().nk_bpe_merge(self.h, i, C.byref(a), C.byref(b)))
            out.append((a.value, b.value))
        return out

    def _ids(self, fn, data: bytes) -> np.ndarray:
        buf = C.create_string_buffer(data, len(data))
        n = _u64(0)
        cap = max(len(data), 1)
        out = np.empty(cap, dtype=np.uint32)
        _check(fn(self.h, buf, len(data), _ptr(out), cap, C.byref(n)))
        return out[: n.value].copy()

    def encode(self, text: str) -> np.ndarray:
        """Bpe::encode (bpe.rs:252-258): pre-token chunks, then merges."""
        return self._ids(lib().nk_bpe_encode, text.encode("utf-8"))

    def encode_bytes(self, data: bytes) -> np.ndarray:
        """Bpe::encode_bytes (bpe.rs:262-266): no pre-token boundaries."""
        return self._ids(lib().nk_bpe_encode_bytes, bytes(data))

    def decode_bytes(self, ids) -> bytes:
        """Bpe::decode_bytes (bpe.rs:268-279); an out-of-range id raises
        NoeticError (NK_ERR_INVALID) where the reference returns None."""
        ids = _u32a(ids).reshape(-1)
        n = _u64(0)
        # Sized first: with no room the call reports the byte count it needs
        # (an out-of-range id fails before that, leaving the count at 0).
        st = lib().nk_bpe_decode_bytes(self.h, _ptr(ids), ids.size, None, 0, C.byref(n))
        if st == NK_OK:
            return b""
        if n.value == 0:
            _check(st)
        out = C.create_string_buffer(n.value)
        _check(lib().nk_bpe_decode_bytes(self.h, _ptr(ids), ids.size, out, n.value, C.byref(n)))
        return out.raw[: n.value]

    def decode(self, ids) -> str:
        """Bpe::decode (bpe.rs:281-286): lossy UTF-8; "" when an id is out of range."""
        try:
            return self.decode_bytes(ids).decode("utf-8", errors="replace")
        except NoeticError:
            return ""

    def close(self):
        if self.h:
            lib().nk_bpe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_tn(a, b, p: int, m: int, n: int, device: int = 0) -> np.ndarray:
    """tensor.rs:156-198 on the GPU: C[m, n] = A[p, m]^T B[p, n]."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    if a.size != p * m or b.size != p * n:
        raise ValueError("a must hold p * m values and b p * n")
    c = np.empty(m * n, dtype=np.float32)
    _check(lib().nk_gemm_tn(_ptr(a), _ptr(b), _ptr(c), p, m, n, device))
    return c.reshape(m, n)


def dwconv_backward(x, w, go, batch: int, t: int, d: int, k: int, gx=None, gw=None, gb=None, device: int = 0):
    """Op::DwConv backward (autograd.rs:1050-1097) on the GPU: the gradients
    add into copies of gx / gw / gb (zeros when None); returns (gx, gw, gb)."""
    n = batch * t * d
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    go = np.ascontiguousarray(go, dtype=np.float32).reshape(-1)
    if x.size != n or go.size != n or w.size != k * d:
        raise ValueError("x and go must hold batch * t * d values and w k * d")
    gx = np.zeros(n, np.float32) if gx is None else np.array(gx, dtype=np.float32).reshape(-1)
    gw = np.zeros(k * d, np.float32) if gw is None else np.array(gw, dtype=np.float32).reshape(-1)
    gb = np.zeros(d, np.float32) if gb is None else np.array(gb, dtype=np.float32).reshape(-1)
    _check(lib().nk_dwconv_backward(_ptr(x), _ptr(w), _ptr(go), _ptr(gx), _ptr(gw), _ptr(gb), batch, t, d, k,
                                    device))
    return gx, gw, gb


def adamw_step(val, grad, m, v, lr: float, t: int, decay: bool = True, b1: float = 0.9, b2: float = 0.95,
               eps: float = 1e-8, wd: float = 0.0, device: int = 0):
    """AdamW::step (optim.rs:33-72) on the GPU for copies of one parameter
    tensor and its moments; t is the step counter after the increment.
    Returns (val, m, v)."""
    val = np.array(val, dtype=np.float32).reshape(-1)
    m = np.array(m, dtype=np.float32).reshape(-1)
    v = np.array(v, dtype=np.float32).reshape(-1)
    grad = np.ascontiguousarray(grad, dtype=np.float32).reshape(-1)
    if not (grad.size == val.size == m.size == v.size):
        raise ValueError("val, grad, m and v must have the same size")
    cfg = NkAdamwCfg(lr, b1, b2, eps, wd, t, int(decay))
    _check(lib().nk_adamw_step(_ptr(val), _ptr(grad), _ptr(m), _ptr(v), val.size, C.byref(cfg), device))
    return val, m, v


def sample_token(logits: np.ndarray, cfg: SampleCfg, history, rng: np.ndarray, device: int = 0) -> int:
    """infer.rs:228-305 on one logit row (mutated in place); rng [4] u64 updated."""
    assert logits.dtype == np.float32 and logits.flags["C_CONTIGUOUS"]
    assert rng.dtype == np.uint64 and rng.size == 4 and rng.flags["C_CONTIGUOUS"]
    hist = _u32a(history).reshape(-1)
    out = np.zeros(1, dtype=np.uint32)
    _check(lib().nk_sample_token(_ptr(logits), logits.size, C.byref(cfg.c()),
                                 _ptr(hist) if hist.size else None, hist.size, _ptr(rng), _ptr(out), device))
    return int(out[0])


def build() -> str:
    """Compile the CUDA library in-tree (nvcc, sm_100a); returns its path."""
    from . import make_lib

    return make_lib.build()
