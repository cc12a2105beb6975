"""ctypes wrapper of the CPU oracle (``oracle/_build/liboracle.so``).

TEST INFRASTRUCTURE ONLY: the test suite, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` use this module as the checker.  The product
package ``noetic_b200`` never imports it.

The oracle restates the reference's f32 CPU path (rng.rs, nn.rs, model.rs,
tensor.rs, infer.rs, scan.rs, autograd.rs forward ops, ckpt.rs, cli.rs
generate).  Parity status: pinned by the reference's known-answer tests and
property tests; RNG / seeded-init bit-exactness is unpinned (the reference has
no known-answer vectors for it and cannot be built without a Rust toolchain).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class Config(C.Structure):
    _fields_ = [
        ("vocab", C.c_uint64),
        ("d_model", C.c_uint64),
        ("n_layer", C.c_uint64),
        ("expand", C.c_uint64),
        ("conv_k", C.c_uint64),
        ("mlp_mult", C.c_uint64),
        ("eps", C.c_float),
        ("tau_max", C.c_float),
    ]


class RngState(C.Structure):
    _fields_ = [("s", C.c_uint64 * 4), ("spare", C.c_float), ("has_spare", C.c_uint32)]


class SampleCfgC(C.Structure):
    _fields_ = [
        ("temperature", C.c_float),
        ("top_k", C.c_uint64),
        ("top_p", C.c_float),
        ("rep_penalty", C.c_float),
        ("rep_window", C.c_uint64),
        ("greedy", C.c_uint32),
    ]


class SampleInfo(C.Structure):
    _fields_ = [
        ("token", C.c_uint32),
        ("kept", C.c_uint32),
        ("used_below", C.c_uint32),
        ("draw", C.c_double),
        ("total", C.c_double),
        ("cdf_margin", C.c_double),
        ("cut_margin", C.c_double),
        ("top2_margin", C.c_double),
        ("order_margin", C.c_double),
    ]


_F = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_U32 = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_P = C.c_void_p
_u64 = C.c_uint64


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sig = {
            "orc_last_error": (C.c_char_p, []),
            "orc_splitmix64": (_u64, [C.POINTER(_u64)]),
            "orc_rng_new": (None, [C.POINTER(RngState), _u64]),
            "orc_rng_next_u64": (_u64, [C.POINTER(RngState)]),
            "orc_rng_f32_unit": (C.c_float, [C.POINTER(RngState)]),
            "orc_rng_below": (_u64, [C.POINTER(RngState), _u64]),
            "orc_rng_normal": (C.c_float, [C.POINTER(RngState)]),
            "orc_worker_count": (_u64, [_u64, _u64, _u64]),
            "orc_matvec_nt": (None, [_F, _P, _F, _F, _u64, _u64, _u64]),
            "orc_gemm_nt": (None, [_F, _F, _F, _u64, _u64, _u64, _u64]),
            "orc_rms_norm_vec": (None, [_F, _F, C.c_float, _F, _u64]),
            "orc_sigmoid": (C.c_float, [C.c_float]),
            "orc_silu": (C.c_float, [C.c_float]),
            "orc_softmax_inplace": (None, [_F, _u64]),
            "orc_argmax": (_u64, [_F, _u64]),
            "orc_scan_sequential": (None, [_F, _F, _F, _u64, _u64, _u64, _u64]),
            "orc_scan_chunked": (None, [_F, _F, _F, _u64, _u64, _u64, _u64]),
            "orc_scan_adjoint": (None, [_F, _F, _F, _u64, _u64, _u64]),
            "orc_gemm_tn": (None, [_F, _F, _F, _u64, _u64, _u64]),
            "orc_dwconv_backward": (None, [_F, _F, _F, _P, _P, _P, _u64, _u64, _u64, _u64]),
            "orc_adamw_step": (C.c_int, [_F, _F, _F, _F, _u64, C.c_float, C.c_float, C.c_float, C.c_float,
                                         C.c_float, _u64, C.c_int]),
            "orc_config_check": (C.c_int, [C.POINTER(Config)]),
            "orc_model_new": (_P, [C.POINTER(Config), C.POINTER(RngState)]),
            "orc_model_free": (None, [_P]),
            "orc_model_tensor_count": (_u64, [_P]),
            "orc_model_tensor_name": (C.c_char_p, [_P, _u64]),
            "orc_model_tensor_rank": (_u64, [_P, _u64]),
            "orc_model_tensor_dim": (_u64, [_P, _u64, _u64]),
            "orc_model_tensor_data": (C.POINTER(C.c_float), [_P, _u64]),
            "orc_model_tensor_numel": (_u64, [_P, _u64]),
            "orc_model_set_threads": (None, [_P, _u64]),
            "orc_lm_logits": (C.c_int, [_P, _U32, _u64, _u64, C.c_int, _F]),
            "orc_softmax_ce": (C.c_int, [_F, _u64, _u64, _U32, C.POINTER(C.c_float)]),
            "orc_lm_loss": (C.c_int, [_P, _U32, _U32, _u64, _u64, C.c_int, C.POINTER(C.c_float), C.c_void_p]),
            "orc_lm_prefill_state": (C.c_int, [_P, _U32, _u64, _u64, _F, _U32, _F]),
            "orc_state_new": (_P, [_P]),
            "orc_state_free": (None, [_P]),
            "orc_state_reset": (None, [_P]),
            "orc_state_numel": (_u64, [_P]),
            "orc_state_get": (None, [_P, _F, C.POINTER(C.c_uint32)]),
            "orc_state_set": (None, [_P, _F, C.c_uint32]),
            "orc_step": (C.c_int, [_P, _P, C.c_uint32, _F]),
            "orc_sample_token": (
                C.c_uint32,
                [_F, _u64, C.POINTER(SampleCfgC), _P, _u64, C.POINTER(RngState), C.POINTER(SampleInfo)],
            ),
            "orc_generate": (
                C.c_int,
                [_P, _U32, _u64, _u64, C.POINTER(SampleCfgC), C.POINTER(RngState), _U32],
            ),
            "orc_crc32": (C.c_uint32, [C.c_char_p, _u64]),
            "orc_ckpt_save": (C.c_int, [_P, C.c_char_p, _P, _P, _u64]),
            "orc_ckpt_load_model": (_P, [C.c_char_p, C.POINTER(RngState)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().orc_last_error().decode()


# ------------------------------------------------------------------ rng.rs
class Rng:
    """rng.rs:17-109 (xoshiro256++ seeded by SplitMix64; Marsaglia normal)."""

    def __init__(self, seed: int = 0, state=None):
        self.st = RngState()
        if state is None:
            lib().orc_rng_new(C.byref(self.st), C.c_uint64(seed))
        else:
            for i in range(4):
                self.st.s[i] = int(state[i])

    @property
    def s(self):
        return [int(self.st.s[i]) for i in range(4)]

    def next_u64(self) -> int:
        return int(lib().orc_rng_next_u64(C.byref(self.st)))

    def f32_unit(self) -> float:
        return float(lib().orc_rng_f32_unit(C.byref(self.st)))

    def below(self, n: int) -> int:
        return int(lib().orc_rng_below(C.byref(self.st), n))

    def normal(self) -> float:
        return float(lib().orc_rng_normal(C.byref(self.st)))


# ------------------------------------------------------------------ model.rs
@dataclass
class LmConfig:
    """model.rs:20-30."""

    vocab: int
    d_model: int = 128
    n_layer: int = 2
    expand: int = 2
    conv_k: int = 4
    mlp_mult: int = 3
    eps: float = 1e-5
    tau_max: float = 128.0

    def c(self) -> Config:
        return Config(self.vocab, self.d_model, self.n_layer, self.expand, self.conv_k,
                      self.mlp_mult, self.eps, self.tau_max)

    def inner(self) -> int:
        return self.d_model * self.expand

    def hidden(self) -> int:
        return self.d_model * self.mlp_mult


@dataclass
class SampleCfg:
    """infer.rs:211-225."""

    temperature: float = 0.9
    top_k: int = 40
    top_p: float = 0.95
    rep_penalty: float = 1.1
    rep_window: int = 64
    greedy: bool = False

    def c(self) -> SampleCfgC:
        return SampleCfgC(self.temperature, self.top_k, self.top_p, self.rep_penalty,
                          self.rep_window, 1 if self.greedy else 0)


class Model:
    """Lm::new (model.rs:183-206) with its named tensors, creation order."""

    def __init__(self, cfg: LmConfig, rng: Rng | None = None, seed: int = 0, _ptr=None):
        self.cfg = cfg
        if _ptr is not None:
            self.ptr = _ptr
        else:
            rng = rng if rng is not None else Rng(seed)
            self.ptr = lib().orc_model_new(C.byref(cfg.c()), C.byref(rng.st))
            if not self.ptr:
                raise ValueError(last_error())

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().orc_model_free(self.ptr)
            self.ptr = None

    def set_threads(self, n: int):
        lib().orc_model_set_threads(self.ptr, n)

    def tensors(self):
        """[(name, ndarray view)] in creation (= checkpoint) order."""
        L = lib()
        out = []
        for i in range(L.orc_model_tensor_count(self.ptr)):
            name = L.orc_model_tensor_name(self.ptr, i).decode()
            rank = L.orc_model_tensor_rank(self.ptr, i)
            shape = tuple(L.orc_model_tensor_dim(self.ptr, i, a) for a in range(rank))
            n = L.orc_model_tensor_numel(self.ptr, i)
            data = L.orc_model_tensor_data(self.ptr, i)
            arr = np.ctypeslib.as_array(data, shape=(n,)).reshape(shape)
            out.append((name, arr))
        return out

    def logits(self, ids: np.ndarray, batch: int, t: int, scan_policy: int = 1) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.empty((batch * t, self.cfg.vocab), dtype=np.float32)
        if lib().orc_lm_logits(self.ptr, ids, batch, t, scan_policy, out) != 0:
            raise ValueError(last_error())
        return out

    def loss(self, ids: np.ndarray, targets: np.ndarray, batch: int, t: int, scan_policy: int = 1,
             want_logits: bool = False):
        """Lm::loss (model.rs:228-234): mean cross-entropy in nats over rows whose
        target is not 0xFFFFFFFF; returns loss, or (loss, logits) with want_logits."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
        targets = np.ascontiguousarray(targets, dtype=np.uint32).reshape(-1)
        out = np.empty((batch * t, self.cfg.vocab), dtype=np.float32) if want_logits else None
        loss = C.c_float()
        if lib().orc_lm_loss(self.ptr, ids, targets, batch, t, scan_policy, C.byref(loss),
                             out.ctypes.data if out is not None else None) != 0:
            raise ValueError(last_error())
        return (float(loss.value), out) if want_logits else float(loss.value)

    def prefill_state(self, ids: np.ndarray, batch: int, t: int):
        """Batched forward; returns (state [batch, L, (k+1)E], heads [batch], last logits)."""
        c = self.cfg
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        st = np.empty((batch, c.n_layer, (c.conv_k + 1) * c.inner()), dtype=np.float32)
        heads = np.empty(batch, dtype=np.uint32)
        last = np.empty((batch, c.vocab), dtype=np.float32)
        if lib().orc_lm_prefill_state(self.ptr, ids, batch, t, st, heads, last) != 0:
            raise ValueError(last_error())
        return st, heads, last

    def save(self, path: str, meta: dict | None = None):
        meta = meta if meta is not None else self.default_meta()
        keys = [k.encode() for k in meta]
        vals = [str(v).encode() for v in meta.values()]
        ka = (C.c_char_p * len(keys))(*keys)
        va = (C.c_char_p * len(vals))(*vals)
        if lib().orc_ckpt_save(self.ptr, path.encode(), C.cast(ka, C.c_void_p),
                               C.cast(va, C.c_void_p), len(keys)) != 0:
            raise IOError(last_error())

    def default_meta(self) -> dict:
        c = self.cfg
        return {"vocab": c.vocab, "d_model": c.d_model, "n_layer": c.n_layer, "expand": c.expand,
                "conv_k": c.conv_k, "mlp_mult": c.mlp_mult, "eps": repr(float(c.eps)),
                "tau_max": repr(float(c.tau_max))}

    @staticmethod
    def load(path: str, rng: Rng | None = None) -> "Model":
        rng = rng if rng is not None else Rng(99)
        ptr = lib().orc_ckpt_load_model(path.encode(), C.byref(rng.st))
        if not ptr:
            raise IOError(last_error())
        # The config is read back from the tensors' shapes.
        L = lib()
        names = [L.orc_model_tensor_name(ptr, i).decode() for i in range(L.orc_model_tensor_count(ptr))]
        emb_v = L.orc_model_tensor_dim(ptr, 0, 0)
        d = L.orc_model_tensor_dim(ptr, 0, 1)
        n_layer = sum(1 for n in names if n.endswith(".n1.gain"))
        e3 = L.orc_model_tensor_dim(ptr, 2, 0)
        k = L.orc_model_tensor_dim(ptr, 4, 0)
        h2 = L.orc_model_tensor_dim(ptr, 9, 0)
        cfg = LmConfig(emb_v, d, n_layer, e3 // 3 // d, k, h2 // 2 // d)
        return Model(cfg, _ptr=ptr)


class Decoder:
    """infer.rs:80-104: Decoder::new / reset / step / state."""

    def __init__(self, model: Model):
        self.model = model
        self.ptr = lib().orc_state_new(model.ptr)
        self.logits = np.zeros(model.cfg.vocab, dtype=np.float32)

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().orc_state_free(self.ptr)
            self.ptr = None

    def reset(self):
        lib().orc_state_reset(self.ptr)

    def step(self, token: int) -> np.ndarray:
        if lib().orc_step(self.model.ptr, self.ptr, int(token), self.logits) != 0:
            raise ValueError(last_error())
        return self.logits

    def get_state(self):
        c = self.model.cfg
        out = np.empty((c.n_layer, (c.conv_k + 1) * c.inner()), dtype=np.float32)
        head = C.c_uint32()
        lib().orc_state_get(self.ptr, out, C.byref(head))
        return out, int(head.value)

    def set_state(self, st: np.ndarray, head: int):
        lib().orc_state_set(self.ptr, np.ascontiguousarray(st, dtype=np.float32), head)


def sample_token(logits: np.ndarray, cfg: SampleCfg, history, rng: Rng, info: bool = False):
    """infer.rs:228-305.  Mutates ``logits`` in place like the reference."""
    assert logits.dtype == np.float32 and logits.flags["C_CONTIGUOUS"]
    hist = np.ascontiguousarray(np.asarray(history, dtype=np.uint32))
    inf = SampleInfo()
    tok = lib().orc_sample_token(logits, logits.size, C.byref(cfg.c()),
                                 hist.ctypes.data if hist.size else None, hist.size,
                                 C.byref(rng.st), C.byref(inf))
    return (int(tok), inf) if info else int(tok)


def generate(model: Model, prompt, n: int, cfg: SampleCfg, rng: Rng) -> np.ndarray:
    """cli.rs:470-518 generate() on token ids."""
    p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
    out = np.zeros(n, dtype=np.uint32)
    if lib().orc_generate(model.ptr, p, p.size, n, C.byref(cfg.c()), C.byref(rng.st), out) != 0:
        raise ValueError(last_error())
    return out


# ------------------------------------------------------------------ tensor.rs / scan.rs
def worker_count(requested: int, jobs: int, total: int) -> int:
    return int(lib().orc_worker_count(requested, jobs, total))


def scan_adjoint(a: np.ndarray, g: np.ndarray, batch: int, t: int, d: int) -> np.ndarray:
    """scan_adjoint (scan.rs:235-260): c_t = g_t + a_{t+1} c_{t+1}, c_T = 0."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    g = np.ascontiguousarray(g, dtype=np.float32).reshape(-1)
    c = np.empty_like(a)
    lib().orc_scan_adjoint(a, g, c, batch, t, d)
    return c


def gemm_tn(a: np.ndarray, b: np.ndarray, p: int, m: int, n: int) -> np.ndarray:
    """gemm_tn (tensor.rs:156-198): C[m,n] = A[p,m]^T B[p,n]."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    c = np.empty(m * n, dtype=np.float32)
    lib().orc_gemm_tn(a, b, c, p, m, n)
    return c.reshape(m, n)


def dwconv_backward(x, w, go, batch: int, t: int, d: int, k: int, gx=None, gw=None, gb=None):
    """Op::DwConv backward (autograd.rs:1050-1097).  Gradients accumulate
    into copies of gx / gw / gb (zeros when None); returns (gx, gw, gb)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    go = np.ascontiguousarray(go, dtype=np.float32).reshape(-1)
    gx = np.zeros(batch * t * d, np.float32) if gx is None else np.array(gx, dtype=np.float32).reshape(-1)
    gw = np.zeros(k * d, np.float32) if gw is None else np.array(gw, dtype=np.float32).reshape(-1)
    gb = np.zeros(d, np.float32) if gb is None else np.array(gb, dtype=np.float32).reshape(-1)
    lib().orc_dwconv_backward(x, w, go, gx.ctypes.data, gw.ctypes.data, gb.ctypes.data, batch, t, d, k)
    return gx, gw, gb


def adamw_step(val, grad, m, v, lr: float, t: int, decay: bool = True, b1: float = 0.9, b2: float = 0.95,
               eps: float = 1e-8, wd: float = 0.0):
    """AdamW::step (optim.rs:33-72) on copies of one parameter tensor and its
    moments; t is the step counter after the increment.  Returns (val, m, v)."""
    val = np.array(val, dtype=np.float32).reshape(-1)
    m = np.array(m, dtype=np.float32).reshape(-1)
    v = np.array(v, dtype=np.float32).reshape(-1)
    grad = np.ascontiguousarray(grad, dtype=np.float32).reshape(-1)
    if lib().orc_adamw_step(val, grad, m, v, val.size, lr, b1, b2, eps, wd, t, int(decay)) != 0:
        raise ValueError(last_error())
    return val, m, v


def softmax_ce(logits: np.ndarray, targets: np.ndarray) -> float:
    """Graph::softmax_ce forward (autograd.rs:579-624) over logits [rows, vocab]."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    targets = np.ascontiguousarray(targets, dtype=np.uint32).reshape(-1)
    loss = C.c_float()
    if lib().orc_softmax_ce(logits, logits.shape[0], logits.shape[1], targets, C.byref(loss)) != 0:
        raise ValueError(last_error())
    return float(loss.value)


def softmax_inplace(x: np.ndarray):
    lib().orc_softmax_inplace(x, x.size)


def argmax(x: np.ndarray) -> int:
    return int(lib().orc_argmax(np.ascontiguousarray(x, dtype=np.float32), x.size))


def sigmoid(x: float) -> float:
    return float(lib().orc_sigmoid(x))


def silu(x: float) -> float:
    return float(lib().orc_silu(x))


def scan_sequential(a, b, batch, t, d, threads=1) -> np.ndarray:
    h = np.empty(batch * t * d, dtype=np.float32)
    lib().orc_scan_sequential(np.ascontiguousarray(a, np.float32).ravel(),
                              np.ascontiguousarray(b, np.float32).ravel(), h, batch, t, d, threads)
    return h


def scan_chunked(a, b, batch, t, d, threads=1) -> np.ndarray:
    h = np.empty(batch * t * d, dtype=np.float32)
    lib().orc_scan_chunked(np.ascontiguousarray(a, np.float32).ravel(),
                           np.ascontiguousarray(b, np.float32).ravel(), h, batch, t, d, threads)
    return h


def crc32(data: bytes) -> int:
    return int(lib().orc_crc32(data, len(data)))
