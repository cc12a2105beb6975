"""Every C-ABI entry point refuses null handles and null buffers with a
status code, before any device work: the reference reports bad arguments
with panics (infer.rs:116-126, model.rs:78-82), which the ABI turns into
NK_ERR_INVALID instead of a crash.  Runs without a GPU."""

import ctypes as C

import pytest

# Operations on caller buffers: null buffers with non-zero sizes are refused.
OPS = ["nk_scan", "nk_scan_device", "nk_scan_adjoint", "nk_scan_adjoint_device", "nk_gemm_tn",
       "nk_gemm_tn_device", "nk_scan_chunked_noalloc_device", "nk_adamw_step", "nk_adamw_step_device",
       "nk_sample_token", "nk_crc32"]
# A zero-sized request is a no-op that succeeds (gemm_tn with p = 0 gives zeros).
EMPTY_OK = ["nk_scan", "nk_scan_device", "nk_scan_adjoint", "nk_scan_adjoint_device", "nk_gemm_tn",
            "nk_gemm_tn_device", "nk_scan_chunked_noalloc_device"]
# Destroying a null handle is allowed, like free(NULL).
DESTROY = ["nk_model_destroy", "nk_decoder_destroy", "nk_bpe_destroy"]
# Calls on a handle, or that return through an output pointer: null is refused.
HANDLE_CALLS = [
    "nk_device_count", "nk_config_check", "nk_model_create", "nk_model_config", "nk_model_init_random",
    "nk_model_tensor_count", "nk_model_tensor_info", "nk_model_set_tensor", "nk_model_get_tensor",
    "nk_model_load_ckpt", "nk_model_save_ckpt", "nk_model_loss", "nk_decoder_create", "nk_decoder_streams",
    "nk_decoder_reset", "nk_decoder_step", "nk_decoder_prefill", "nk_decoder_sample", "nk_decoder_generate",
    "nk_decoder_get_state", "nk_decoder_set_state", "nk_decoder_step_greedy_device", "nk_decoder_step_greedy",
    "nk_decoder_cuda_stream", "nk_decoder_sync", "nk_decoder_set_engine", "nk_decoder_launch_count",
    "nk_decoder_profile_begin", "nk_decoder_profile_end", "nk_bpe_create_bytes_only", "nk_bpe_load",
    "nk_bpe_save", "nk_bpe_vocab_size", "nk_bpe_merge", "nk_bpe_encode", "nk_bpe_encode_bytes",
    "nk_bpe_decode_bytes"]


def _args(nb, name, size):
    vals = []
    for a in nb.SIGNATURES[name][1]:
        if a in (C.c_void_p, C.c_char_p) or (isinstance(a, type) and issubclass(a, C._Pointer)):
            vals.append(None)
        elif a in (C.c_float, C.c_double):
            vals.append(0.0)
        else:
            vals.append(size)
    return vals


def test_every_declared_call_is_covered(nb):
    covered = set(OPS) | set(DESTROY) | set(HANDLE_CALLS) | {"nk_last_error", "nk_dwconv_backward",
                                                             "nk_dwconv_backward_device"}
    assert covered == set(nb.SIGNATURES)


@pytest.mark.parametrize("name", OPS)
def test_null_buffers_are_refused(nb, name):
    assert getattr(nb.lib(), name)(*_args(nb, name, 1)) == nb.NK_ERR_INVALID
    assert nb.lib().nk_last_error()


@pytest.mark.parametrize("name", EMPTY_OK)
def test_empty_requests_succeed(nb, name):
    assert getattr(nb.lib(), name)(*_args(nb, name, 0)) == 0


def test_dwconv_backward_needs_the_inputs_of_each_requested_gradient(nb):
    L = nb.lib()
    buf = (C.c_float * 8)()
    p = C.cast(buf, C.c_void_p)
    # No gradient requested: nothing to do.
    assert L.nk_dwconv_backward(None, None, None, None, None, None, 1, 1, 1, 1, 0) == 0
    # gb needs go; gx needs w and go; gw needs x and go.
    assert L.nk_dwconv_backward(None, None, None, None, None, p, 1, 1, 1, 1, 0) == nb.NK_ERR_INVALID
    assert L.nk_dwconv_backward(None, None, p, p, None, None, 1, 1, 1, 1, 0) == nb.NK_ERR_INVALID
    assert L.nk_dwconv_backward(None, p, p, None, p, None, 1, 1, 1, 1, 0) == nb.NK_ERR_INVALID


@pytest.mark.parametrize("name", HANDLE_CALLS)
def test_null_handles_and_outputs_are_refused(nb, name):
    assert getattr(nb.lib(), name)(*_args(nb, name, 0)) != 0
    assert nb.lib().nk_last_error()


@pytest.mark.parametrize("name", DESTROY)
def test_destroying_null_is_a_no_op(nb, name):
    assert getattr(nb.lib(), name)(None) == 0


# Sizes whose products would wrap around 64 bits (or exceed 2^37 elements per
# array, more than a device holds) are refused before any device work, rather
# than wrapping to an "empty" request or an undersized allocation.
HUGE = 1 << 33


def test_oversized_requests_are_refused(nb):
    L = nb.lib()
    buf = (C.c_float * 64)()
    p = C.cast(buf, C.c_void_p)
    cfg = nb.NkAdamwCfg(1e-3, 0.9, 0.999, 1e-8, 0.0, 1, 0)
    calls = {
        "scan": lambda: L.nk_scan(p, p, p, HUGE, HUGE, HUGE, 1, 0),
        "scan_device": lambda: L.nk_scan_device(p, p, p, HUGE, HUGE, HUGE, 0, None),
        "scan_adjoint": lambda: L.nk_scan_adjoint(p, p, p, HUGE, HUGE, HUGE, 1, 0),
        "scan_adjoint_device": lambda: L.nk_scan_adjoint_device(p, p, p, 1 << 20, 1 << 20, 1 << 20, 1, None),
        "scan_noalloc": lambda: L.nk_scan_chunked_noalloc_device(p, p, p, HUGE, HUGE, HUGE, None),
        "gemm_tn": lambda: L.nk_gemm_tn(p, p, p, 1 << 40, 1 << 20, 1 << 20, 0),
        "gemm_tn_device": lambda: L.nk_gemm_tn_device(p, p, p, 1 << 61, 4, 4, None),
        "dwconv": lambda: L.nk_dwconv_backward(p, p, p, p, p, p, HUGE, HUGE, 1, 1, 0),
        "dwconv_device": lambda: L.nk_dwconv_backward_device(p, p, p, p, p, p, 1 << 20, 1 << 20, 1 << 20, 1, None),
        "adamw": lambda: L.nk_adamw_step(p, p, p, p, 1 << 62, C.byref(cfg), 0),
        "adamw_device": lambda: L.nk_adamw_step_device(p, p, p, p, (1 << 37) + 1, C.byref(cfg), None),
    }
    for name, call in calls.items():
        assert call() == nb.NK_ERR_INVALID, name
        assert b"2^37" in nb.lib().nk_last_error() or b"limit" in nb.lib().nk_last_error(), name


def test_a_missing_library_fails_loudly(nb, monkeypatch, tmp_path):
    # No CPU fallback: without the built library every product call raises.
    import numpy as np

    monkeypatch.setattr(nb, "LIB_PATH", str(tmp_path / "libnoetic_gpu.so"))
    monkeypatch.setattr(nb, "_lib", None)
    with pytest.raises(nb.NoeticError) as e:
        nb.lib()
    assert e.value.status == nb.NK_ERR_UNSUPPORTED
    with pytest.raises(nb.NoeticError):
        nb.scan_chunked(np.ones(4, np.float32), np.ones(4, np.float32), 1, 4, 1)
