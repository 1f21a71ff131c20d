"""ctypes binding of libspeckv.so (the C ABI declared in include/speckv.h).

The library is loaded on first use. A missing library is an error, never a
silent fallback: build it with ``python -m analysis_spec_b200.build``.
"""
import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name('libspeckv.so')

SPECKV_OK, SPECKV_EINVAL, SPECKV_ECUDA, SPECKV_ENOSUPPORT = 0, 1, 2, 3
MAX_LAYERS = 64
F32, BF16, F16 = 0, 1, 2

DEVICE_ERROR_KINDS = {1: 'remap index', 2: 'compact index', 3: 'move index', 4: 'tree parent index',
                      5: 'padding owner index', 6: 'wait timeout', 7: 'scheduling packet',
                      8: 'seen index', 9: 'history index', 10: 'row table'}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_pi64 = ctypes.POINTER(ctypes.c_int64)
_pp = ctypes.POINTER(ctypes.c_void_p)

# name -> argtypes (every function returns int status)
SIGNATURES = {
    'speckv_append_rows': [_pp, _pp, _pp, _pp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _i32, _p,
                           _i64, _p],
    'speckv_append_commit_rows': [_pp, _pp, _pp, _pp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _i32,
                                  _p, _i64, _i64, _i64, _i64, _i64, _p],
    'speckv_compact_suffix': [_pp, _pp, _i32, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i32,
                              _p, _i64, _p],
    'speckv_commit_round': [_pp, _pp, _i32, _i64, _i64, _i64, _i64, _i64, _i32, _p, _i64, _i64, _i64, _p, _i64, _i64,
                            _p, _i64, _i64, _p, _p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _p],
    'speckv_remap_rows': [_pp, _pp, _i32, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i32, _p],
    'speckv_remap_rows_static': [_pp, _pp, _i32, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _p],
    'speckv_move_rows': [_pp, _pp, _i32, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _p],
    'speckv_pack_tree': [_p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _p],
    'speckv_trace_path': [_p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _p, _p],
    'speckv_pad_verified_path': [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i64,
                                 _i64, _p, _i64, _p],
    'speckv_pad_schedule': [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p,
                            _i64, _p, _i64, _i64, _p, _p],
    'speckv_tree_mask': [_p, _i64, _i64, _i64, _i64, _p, _i32, _p, _i64, _p],
    'speckv_position_update': [_p, _i64, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _p, _p],
    'speckv_tree_mask_bits': [_p, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _p, _p],
    'speckv_tree_attention_bits': [_p, _pi64, _p, _pi64, _p, _pi64, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                   _i64, ctypes.c_float, _i32, _p, _i64, _p],
    'speckv_tree_attention': [_p, _pi64, _p, _pi64, _p, _pi64, _p, _i32, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                              ctypes.c_float, _i32, _p],
    'speckv_tree_attention_bits_append': [_p, _pi64, _p, _pi64, _p, _pi64, _i64, _i64, _p, _pi64, _p, _pi64, _p,
                                          _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _i32, _p],
    'speckv_device_error': [ctypes.POINTER(ctypes.c_uint64), _p],
    'speckv_plan_launch': [_p, _p],
    'speckv_causal_mask': [_p, _i32, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _p],
    'speckv_history_append': [_i32, _pp, _pi64, _pp, _pi64, _pp, _pi64, _pp, _pi64, _pi64, _pi64, _pi64, _pi64,
                              _p, _p, _i64, _i64, _p],
    'speckv_mask_bits': [_p, _i32, _i64, _i64, _i64, _pi64, _p, _i64, _p, _p, _p],
    'speckv_history_pack': [_p, _p, _i64, _i64, _i64, _p, _i64, _i64, _p],
    'speckv_expansion_mask': [_p, _i32, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _p],
    'speckv_version': [],
    'speckv_attention_launches': [_pi64, _pi64],
    'speckv_attention_test_hooks': [_i64, _i32],
    'speckv_acceptance_counts': [_p, _i64, _i64, _i64, _p, _p],
    'speckv_attention_set_ctas': [_i32],
    'speckv_attention_set_chunks': [_i32],
}

# entries with a prepare / launch split (speckv_<name>_prepare + speckv_plan_launch)
PREPARED = ('speckv_append_rows', 'speckv_commit_round', 'speckv_append_commit_rows')

_lock = threading.Lock()
_lib = None


def load():
    """Returns the loaded library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f'{LIB_PATH.name} is not built; run `python -m analysis_spec_b200.build` '
                                   '(the CUDA path has no fallback)')
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_int
            lib.speckv_last_error.argtypes = []
            lib.speckv_last_error.restype = ctypes.c_char_p
            lib.speckv_remap_scratch_bytes.argtypes = [_i64, _i64, _i64, _i64, _i32]
            lib.speckv_remap_scratch_bytes.restype = ctypes.c_int64
            for name in PREPARED:  # same arguments without the stream, then the plan out-pointer
                fn = getattr(lib, name + '_prepare')
                fn.argtypes = SIGNATURES[name][:-1] + [_pp]
                fn.restype = ctypes.c_int
            lib.speckv_plan_release.argtypes = [_p]
            lib.speckv_plan_release.restype = None
            _lib = lib
    return _lib


class SpecKVError(RuntimeError):
    """A libspeckv call returned a non-zero status."""

    def __init__(self, name, status, message):
        super().__init__(f'{name} failed (status {status}): {message}')
        self.status = status


class _Profile:
    """Optional per-entry-point CUDA-event timing and call counting (off by default)."""
    enabled = False
    calls = 0
    events = {}  # name -> list of (start, end) torch.cuda.Event

    @classmethod
    def reset(cls):
        cls.calls = 0
        cls.events = {}


profile = _Profile


def call(name, *args):
    """Calls entry point `name`; kernels launch on the stream passed as its last argument,
    which the _ops front end takes from torch's current stream (where profiling events go)."""
    lib = load()
    if profile.enabled and name != 'speckv_device_error':
        import torch
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        status = getattr(lib, name)(*args)
        end.record()
        profile.events.setdefault(name, []).append((start, end))
    else:
        status = getattr(lib, name)(*args)
    profile.calls += 1
    if status != SPECKV_OK:
        raise SpecKVError(name, status, lib.speckv_last_error().decode(errors='replace'))


class Plan:
    """A prepared launch of entry point `name` (see speckv_plan_launch); freed with the object.
    It launches with the GPU it was prepared on current (the C side refuses any other)."""

    def __init__(self, name, handle, stream, device):
        self.name, self.handle, self.stream, self.device = name, handle, stream, device

    def __call__(self):
        """Enqueues the prepared kernel (profiled under the entry point's own name)."""
        if self.device >= 0:
            import torch
            if torch.cuda.current_device() != self.device:
                with torch.cuda.device(self.device):
                    return self._launch()
        return self._launch()

    def _launch(self):
        lib = load()
        if profile.enabled:
            import torch
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            status = lib.speckv_plan_launch(self.handle, self.stream)
            end.record()
            profile.events.setdefault(self.name, []).append((start, end))
        else:
            status = lib.speckv_plan_launch(self.handle, self.stream)
        profile.calls += 1
        if status != SPECKV_OK:
            raise SpecKVError(self.name, status, lib.speckv_last_error().decode(errors='replace'))

    def __del__(self):
        if self.handle and _lib is not None:
            _lib.speckv_plan_release(self.handle)
            self.handle = None


def prepare(name, *args):
    """speckv_<name>_prepare with the entry point's arguments (the last one, the stream,
    is kept for the launch); returns a Plan."""
    lib = load()
    handle = ctypes.c_void_p()
    status = getattr(lib, name + '_prepare')(*args[:-1], ctypes.byref(handle))
    if status != SPECKV_OK:
        raise SpecKVError(name + '_prepare', status, lib.speckv_last_error().decode(errors='replace'))
    import torch
    return Plan(name, handle, args[-1], torch.cuda.current_device() if torch.cuda.is_available() else -1)


def ptr_array(values):
    return (ctypes.c_void_p * len(values))(*values)


def i64_array(values):
    return (ctypes.c_int64 * len(values))(*values)
