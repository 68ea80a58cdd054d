"""ctypes binding of ``libblitzgs_b200.so`` (C ABI in include/blitzgs_b200.h).

The library is loaded from the package's ``lib/`` directory.  There is no
fallback: if the library is missing or a call fails, a RuntimeError is raised.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libblitzgs_b200.so")

_i32, _i64, _f32, _vp, _sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/blitzgs_b200.h
SIGNATURES = {
    "blitz_version": (ctypes.c_char_p, []),
    "blitz_last_error": (ctypes.c_char_p, []),
    "blitz_preprocess_forward": (_i32, [
        _i64, _i32, _i32, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _f32, _vp, _vp, _vp, _f32, _f32,
        _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_rasterize_count": (_i32, [_i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_rasterize_bin": (_i32, [_i64, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp,
                                   _vp]),
    "blitz_rasterize_blend": (_i32, [_i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                     _vp]),
    "blitz_rasterize_depth": (_i32, [_i64, _i32, _i32] + [_vp] * 18),
    "blitz_mark_visible": (_i32, [_i64, _vp, _vp, _vp, _vp, _vp]),
    "blitz_preprocess_backward": (_i32, [
        _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _f32, _vp, _vp, _vp, _f32, _f32,
        _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _vp]),
    "blitz_preprocess_forward_raw": (_i32, [
        _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _f32, _vp, _vp, _vp, _f32, _f32,
        _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "blitz_preprocess_scratch_bytes": (_sz, [_i64]),
    "blitz_exchange_pack_scratch_bytes": (_sz, [_i64, _i32]),
    "blitz_preprocess_batch_scratch_bytes": (_sz, [_i32, _i64]),
    "blitz_exchange_pack": (_i32, [_i64, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _sz, _vp]),
    "blitz_exchange_pack_batch": (_i32, [_i32, _i32, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "blitz_preprocess_forward_raw_batch": (_i32, [
        _i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _f32, _vp, _vp, _vp, _vp, _i32, _i32,
        _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "blitz_preprocess_backward_raw_batch": (_i32, [
        _i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _f32,
        _vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp]),
    "blitz_get_local2j_ids_bool_adjust_mode6": (_i32, [_i32, _i32, _i32, _i32, _i64, _vp, _vp, _vp, _i32, _vp,
                                                        _vp]),
    "blitz_adam_update": (_i32, [_vp, _vp, _vp, _vp, _vp, _f32, _f32, _f32, _f32, _i64, _i64, _vp]),
    "blitz_adam_update_rows": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _f32, _f32, _f32, _f32, _f32, _i64, _i64,
                                      _vp]),
    "blitz_preprocess_backward_raw": (_i32, [
        _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _f32, _vp, _vp, _vp, _f32,
        _f32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
        _i64, _vp, _i64, _i32, _i32, _vp]),
    "blitz_render_count": (_i32, [_i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_render_scratch_bytes": (_sz, [_i64, _i64, _i64, _i32, _i32]),
    "blitz_render_forward": (_i32, [
        _i64, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp,
        _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_render_bin": (_i32, [_i64, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp]),
    "blitz_render_blend": (_i32, [_i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                  _vp, _vp, _vp, _vp, _vp]),
    "blitz_render_bin_noalloc": (_i32, [_i64, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_render_backward": (_i32, [
        _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_loss_forward": (_i32, [_i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_loss_backward": (_i32, [_i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_get_local2j_ids_bool": (_i32, [_i32, _i32, _i32, _i32, _i64, _vp, _vp, _vp, _i32, _vp, _vp]),
    "blitz_fp32_probe": (_i32, [_i32, _i64, _vp, _vp]),
    "blitz_loss_combine": (_i32, [_vp, _vp, _f32, _f32, _f32, _f32, _vp, _vp]),
    "blitz_loss_combine_backward": (_i32, [_vp, _vp, _vp, _vp, _f32, _f32, _f32, _f32, _vp, _vp]),
    "blitz_read_totals": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_zero_fill_async": (_i32, [_i32, _vp, _vp, _vp]),
    "blitz_zero_fill_wait": (_i32, [_vp]),
    "blitz_zero_rows": (_i32, [_i32, _vp, _vp, _vp, _i64, _vp]),
    "blitz_exchange_unpack": (_i32, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "blitz_grad_records_pack": (_i32, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load (once) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"blitzgs_b200 native library not found at {LIB_PATH}; build it with "
                "`python -m blitzgs_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols():
    return list(SIGNATURES)


def call(name, *args):
    """Call an int-returning entry point; raise RuntimeError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.blitz_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed ({rc}): {msg}")
    return rc


def ptr(t):
    """Device pointer of a tensor as an int (None -> NULL); ctypes converts it
    for the void* parameters."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None):
    """cudaStream_t (as an int) of ``stream``, else of the current device's
    current stream.  The default path asks torch's C accessors directly:
    torch.cuda.current_stream() builds a Stream object and re-resolves the
    device on every call (~15 us, several times per training step)."""
    import torch
    if stream is not None:
        return stream.cuda_stream
    return torch._C._cuda_getCurrentRawStream(torch._C._cuda_getDevice())
