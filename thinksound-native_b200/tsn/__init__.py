"""ctypes binding of the C ABI in include/tsn.h (libtsn.so, built in this directory).

The classes mirror the reference's C++ faces: :class:`Device` is ``tn::gpu::Device``
(src/gpu.h), its runtime methods are ``tn::Runtime`` (src/net.h), and :class:`Dit` is
``tn::DitModel`` (src/models.h) plus the sampler loop of src/pipeline.cpp. Every call raises
:class:`TsnError` on a non-zero status. There is no CPU path: without the library or an sm_100
device the calls fail.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtsn.so")

TSN_COMPUTE_F16 = 0
TSN_COMPUTE_BF16 = 1

_ERRS = {1: "ARG", 2: "CUDA", 3: "IO", 4: "FORMAT", 5: "MISSING", 6: "OOM", 7: "UNSUPPORTED",
         8: "TIMEOUT", 9: "STATE"}


class TsnError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"TSN_ERR_{_ERRS.get(code, code)}: {msg}")
        self.code = code


class Geom(C.Structure):
    _fields_ = [("H", C.c_uint32), ("NH", C.c_uint32), ("F", C.c_uint32), ("depth", C.c_uint32),
                ("fused_depth", C.c_uint32), ("latent_dim", C.c_uint32), ("rope_theta", C.c_float),
                ("t_max_period", C.c_float)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


def geom(H=1024, NH=16, F=4096, depth=21, fused_depth=14, latent_dim=64, rope_theta=10000.0,
         t_max_period=1.0) -> Geom:
    return Geom(H, NH, F, depth, fused_depth, latent_dim, rope_theta, t_max_period)


_lib = None

# (name, restype, argtypes)
_SIGS = [
    ("tsn_last_error", C.c_char_p, []),
    ("tsn_version", C.c_int, []),
    ("tsn_device_create", C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    ("tsn_device_destroy", C.c_int, [C.c_void_p]),
    ("tsn_device_set_stream", C.c_int, [C.c_void_p, C.c_void_p]),
    ("tsn_device_stream", C.c_void_p, [C.c_void_p]),
    ("tsn_alloc", C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
    ("tsn_wrap", C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
    ("tsn_begin", C.c_int, [C.c_void_p]),
    ("tsn_dispatch", C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                               C.POINTER(C.c_void_p), C.c_int, C.c_void_p, C.c_size_t]),
    ("tsn_commit", C.c_int, [C.c_void_p]),
    ("tsn_exec_width", C.c_uint32, [C.c_void_p, C.c_char_p]),
    ("tsn_last_gpu_ms", C.c_double, [C.c_void_p]),
    ("tsn_selftest_device_timeout", C.c_int, [C.c_void_p, C.c_uint32]),
    ("tsn_selftest_gemm_lo8", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
                                        C.c_uint32, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.POINTER(C.c_float)]),
    ("tsn_selftest_gemv_jobs", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.POINTER(C.c_uint32), C.c_int, C.c_uint32, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_int]),
    ("tsn_gemm", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                           C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    ("tsn_gemm_noalloc", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    ("tsn_gemv", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
                           C.c_uint32, C.c_uint32, C.c_int]),
    ("tsn_conv", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                           C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                           C.c_uint32, C.c_uint32, C.c_int]),
    ("tsn_silu", C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    ("tsn_copy", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    ("tsn_swiglu", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    ("tsn_add", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    ("tsn_add_bcast_col", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32]),
    ("tsn_cfg_euler", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_float, C.c_float]),
    ("tsn_mean_cols", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32]),
    ("tsn_dit_load", C.c_int, [C.c_void_p, C.c_char_p, C.c_int, C.POINTER(C.c_void_p)]),
    ("tsn_dit_inspect", C.c_int, [C.c_char_p, C.POINTER(Geom), C.POINTER(C.c_size_t)]),
    ("tsn_dit_load_synthetic", C.c_int, [C.c_void_p, C.POINTER(Geom), C.c_uint64, C.c_int, C.POINTER(C.c_void_p)]),
    ("tsn_dit_free", C.c_int, [C.c_void_p]),
    ("tsn_vae_load", C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
    ("tsn_vae_load_synthetic", C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64,
                                         C.POINTER(C.c_void_p)]),
    ("tsn_vae_decode", C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32)]),
    ("tsn_vae_last_ms", C.c_double, [C.c_void_p]),
    ("tsn_vae_profile_ops", C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    ("tsn_vae_flops", C.c_double, [C.c_void_p]),
    ("tsn_vae_launches", C.c_int, [C.c_void_p]),
    ("tsn_vae_free", C.c_int, [C.c_void_p]),
    ("tsn_t5_load", C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
    ("tsn_clip_load", C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
    ("tsn_encoder_info", C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    ("tsn_encoder_encode", C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]),
    ("tsn_encoder_last_ms", C.c_double, [C.c_void_p]),
    ("tsn_encoder_flops", C.c_double, [C.c_void_p]),
    ("tsn_encoder_launches", C.c_int, [C.c_void_p]),
    ("tsn_encoder_weight_bytes", C.c_double, [C.c_void_p]),
    ("tsn_encoder_profile_ops", C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    ("tsn_encoder_free", C.c_int, [C.c_void_p]),
    ("tsn_gguf_write_synthetic_t5", C.c_int, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]),
    ("tsn_gguf_write_synthetic_clip", C.c_int, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]),
    ("tsn_dit_get_geom", C.c_int, [C.c_void_p, C.POINTER(Geom)]),
    ("tsn_dit_weight_bytes", C.c_size_t, [C.c_void_p]),
    ("tsn_dit_prepare", C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    ("tsn_dit_set_conditioning", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("tsn_dit_set_x", C.c_int, [C.c_void_p, C.c_void_p]),
    ("tsn_dit_get_x", C.c_int, [C.c_void_p, C.c_void_p]),
    ("tsn_dit_forward", C.c_int, [C.c_void_p, C.c_float, C.c_void_p]),
    ("tsn_dit_forward_taps", C.c_int, [C.c_void_p, C.c_float, C.c_void_p]),
    ("tsn_dit_tap", C.c_int, [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    ("tsn_dit_step", C.c_int, [C.c_void_p, C.c_float, C.c_float, C.c_float]),
    ("tsn_dit_sample", C.c_int, [C.c_void_p, C.c_int, C.c_float]),
    ("tsn_dit_schedule", C.c_int, [C.c_void_p, C.c_int, C.c_float]),
    ("tsn_dit_run_steps", C.c_int, [C.c_void_p, C.c_int]),
    ("tsn_dit_split_schedule", C.c_int, [C.c_void_p, C.c_int]),
    ("tsn_dit_split_forward", C.c_int, [C.c_void_p, C.c_void_p]),
    ("tsn_dit_split_update", C.c_int, [C.c_void_p, C.c_void_p, C.c_float]),
    ("tsn_dit_step_host", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_float, C.c_float]),
    ("tsn_dit_kernels_per_step", C.c_int, [C.c_void_p]),
    ("tsn_dit_profile_step", C.c_int, [C.c_void_p, C.POINTER(C.c_double)]),
    ("tsn_dit_profile_ops", C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    ("tsn_dit_get_conditioning", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("tsn_dit_prep_conditioning", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]),
    ("tsn_dit_prep_text_arm", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("tsn_dit_trace_op", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_int)]),
    ("tsn_dit_timeline", C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_int)]),
    ("tsn_dit_autotune", C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    ("tsn_dit_get_tiles", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
    ("tsn_dit_set_tiles", C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    ("tsn_gguf_write_synthetic", C.c_int, [C.c_char_p, C.POINTER(Geom), C.c_uint64, C.c_int]),
    ("tsn_gguf_write_synthetic_vae", C.c_int, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]),
]

EXPORTED = [s[0] for s in _SIGS]


def lib():
    """Load libtsn.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise TsnError(2, f"{LIB_PATH} not built (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int):
    if rc != 0:
        msg = lib().tsn_last_error()
        raise TsnError(rc, msg.decode() if msg else "")


def _p(x):
    """Address of a torch tensor / numpy array / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(type(x))


class Device:
    """tn::gpu::Device + tn::Runtime over one CUDA device."""

    def __init__(self, ordinal: int = 0, stream: int | None = None):
        h = C.c_void_p()
        check(lib().tsn_device_create(ordinal, C.byref(h)))
        self.h = h
        self._models = weakref.WeakSet()   # models must be freed before their device
        if stream is not None:
            check(lib().tsn_device_set_stream(self.h, C.c_void_p(stream)))

    def close(self):
        if self.h:
            for m in list(self._models):
                m.close()
            lib().tsn_device_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # --- gpu.h Device
    def alloc(self, nbytes: int) -> int:
        p = C.c_void_p()
        check(lib().tsn_alloc(self.h, nbytes, C.byref(p)))
        return p.value

    def dispatch(self, kernel: str, grid, block, bufs, params: bytes = b""):
        g = (C.c_uint32 * 3)(*grid)
        b = (C.c_uint32 * 3)(*block)
        arr = (C.c_void_p * max(1, len(bufs)))(*[_p(x) for x in bufs])
        pb = C.create_string_buffer(params, len(params)) if params else None
        check(lib().tsn_dispatch(self.h, kernel.encode(), g, b, arr, len(bufs), pb, len(params)))

    def commit(self):
        check(lib().tsn_commit(self.h))

    def last_gpu_ms(self) -> float:
        return lib().tsn_last_gpu_ms(self.h)

    def exec_width(self, kernel: str) -> int:
        return lib().tsn_exec_width(self.h, kernel.encode())

    def selftest_timeout(self, limit_us: int = 1000):
        """Run the bounded-wait self-test (a wait nothing completes); raises TsnError (TSN_ERR_TIMEOUT
        expected) unless the wait somehow completed."""
        check(lib().tsn_selftest_device_timeout(self.h, limit_us))

    def selftest_gemm_lo8(self, W, X, Y, bias, M, N, K, wexp, mode, bn, reps=1) -> float:
        """Experimental GEMM with an e4m3 low-order product (mode 0) or the split f16 GEMM (mode 1);
        returns the mean event-timed milliseconds of one launch."""
        ms = C.c_float(0.0)
        check(lib().tsn_selftest_gemm_lo8(self.h, _p(W), _p(X), _p(Y), _p(bias), M, N, K, wexp, mode, bn, reps,
                                          C.byref(ms)))
        return ms.value

    def selftest_gemv_jobs(self, W, bias, x, Y, Ns, K, nb, nb_cap, act=0, blocks=148, tc=False):
        """The step's batched GEMV over several jobs (f16 rows back to back, Y [nb][sum Ns]), on the CUDA
        cores or (tc) the tensor cores; synchronises."""
        arr = (C.c_uint32 * len(Ns))(*Ns)
        check(lib().tsn_selftest_gemv_jobs(self.h, _p(W), _p(bias), _p(x), _p(Y), arr, len(Ns), K, nb, nb_cap,
                                           act, blocks, int(tc)))

    # --- net.h Runtime
    def gemm(self, wf16, W, X, Y, bias, M, N, K, ldx=0, ldw=0, ldy=0):
        check(lib().tsn_gemm(self.h, int(wf16), _p(W), _p(X), _p(Y), _p(bias), M, N, K, ldx, ldw, ldy))

    def gemm_noalloc(self, W, X, Y, bias, M, N, K, ldx=0, ldw=0, ldy=0):
        """tsn_gemm (f16 weights) without any device allocation: scratch is a fixed 8 MiB array."""
        check(lib().tsn_gemm_noalloc(self.h, _p(W), _p(X), _p(Y), _p(bias), M, N, K, ldx, ldw, ldy))

    def gemv(self, W, X, Y, bias, N, K, ldw=0, wf16=True):
        check(lib().tsn_gemv(self.h, _p(W), _p(X), _p(Y), _p(bias), N, K, ldw, int(wf16)))

    def conv(self, wf16, W, bias, x, y, T, OL, IC, OC, K, stride=1, pad=0, dil=1, convt=False):
        check(lib().tsn_conv(self.h, int(wf16), _p(W), _p(bias), _p(x), _p(y), T, OL, IC, OC, K, stride, pad,
                             dil, int(convt)))

    def cfg_euler(self, fc, fu, x, n, cfg, dt):
        check(lib().tsn_cfg_euler(self.h, _p(fc), _p(fu), _p(x), n, cfg, dt))


class Vae:
    """tn::VaeModel's decoder on the device: latent [T, 64] -> audio [T * 2048, out_channels]."""

    def __init__(self, dev: Device, gguf: str | None = None, channels: int = 128, latent_dim: int = 64,
                 out_channels: int = 2, seed: int = 4242):
        self.dev = dev
        h = C.c_void_p()
        if gguf is not None:
            check(lib().tsn_vae_load(dev.h, gguf.encode(), C.byref(h)))
        else:
            check(lib().tsn_vae_load_synthetic(dev.h, latent_dim, channels, out_channels, seed, C.byref(h)))
        self.h = h
        self.out_channels = out_channels
        dev._models.add(self)

    def decode(self, latent):
        """Host latent [T, latent_dim] f32 -> host audio [T_audio, out_channels] f32."""
        import numpy as np
        lat = np.ascontiguousarray(latent, np.float32)
        T = lat.shape[0]
        out = np.zeros((T * 2048, self.out_channels), np.float32)
        ta = C.c_uint32()
        check(lib().tsn_vae_decode(self.h, lat.ctypes.data, T, out.ctypes.data, out.size, C.byref(ta)))
        return out[:ta.value]

    def last_ms(self) -> float:
        return lib().tsn_vae_last_ms(self.h)

    def flops(self) -> float:
        return lib().tsn_vae_flops(self.h)

    def launches(self) -> int:
        """Kernel launches in one decode graph of the last decoded length."""
        return lib().tsn_vae_launches(self.h)

    def profile_ops(self) -> str:
        buf = C.create_string_buffer(1 << 18)
        check(lib().tsn_vae_profile_ops(self.h, buf, len(buf)))
        return buf.value.decode()

    def close(self):
        if self.h and self.dev.h:
            lib().tsn_vae_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Dit:
    """tn::DitModel on the device, with the CFG-batched fast path."""

    def __init__(self, dev: Device, gguf: str | None = None, synthetic: Geom | None = None, seed: int = 4242,
                 compute: int = TSN_COMPUTE_F16):
        self.dev = dev
        h = C.c_void_p()
        if gguf is not None:
            check(lib().tsn_dit_load(dev.h, gguf.encode(), compute, C.byref(h)))
        else:
            g = synthetic or geom()
            check(lib().tsn_dit_load_synthetic(dev.h, C.byref(g), seed, compute, C.byref(h)))
        self.h = h
        dev._models.add(self)
        g = Geom()
        check(lib().tsn_dit_get_geom(self.h, C.byref(g)))
        self.geom = g
        self.T = self.C = self.TS = self.arms = 0

    def close(self):
        if self.h and self.dev.h:
            lib().tsn_dit_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight_bytes(self) -> int:
        return lib().tsn_dit_weight_bytes(self.h)

    def prepare(self, T: int, C_: int, TS: int, arms: int = 2):
        check(lib().tsn_dit_prepare(self.h, T, C_, TS, arms))
        self.T, self.C, self.TS, self.arms = T, C_, TS, arms

    def set_conditioning(self, clip_pp, sync_gather, text_pp, gcmlp):
        check(lib().tsn_dit_set_conditioning(self.h, _p(clip_pp), _p(sync_gather), _p(text_pp), _p(gcmlp)))

    def get_conditioning(self, clip_pp=None, sync_gather=None, text_pp=None, gcmlp=None):
        check(lib().tsn_dit_get_conditioning(self.h, _p(clip_pp), _p(sync_gather), _p(text_pp), _p(gcmlp)))

    def prep_conditioning(self, clip_f, sync_f, sync_S: int):
        """prep_conditioning on the GPU: clip_f [C, 1024], sync_f [sync_S, 768] f32."""
        check(lib().tsn_dit_prep_conditioning(self.h, _p(clip_f), _p(sync_f), sync_S))

    def prep_text_arm(self, arm: int, text_cat, gtext):
        """prep_text_arm on the GPU for CFG arm `arm`: text_cat [TS, 2048], gtext [1024] f32."""
        check(lib().tsn_dit_prep_text_arm(self.h, arm, _p(text_cat), _p(gtext)))

    def set_x(self, x):
        check(lib().tsn_dit_set_x(self.h, _p(x)))

    def get_x(self, out):
        check(lib().tsn_dit_get_x(self.h, _p(out)))

    def forward(self, t: float, flow_out):
        check(lib().tsn_dit_forward(self.h, t, _p(flow_out)))

    def forward_taps(self, t: float, flow_out=None):
        check(lib().tsn_dit_forward_taps(self.h, t, _p(flow_out)))

    def tap(self, name: str, arm: int = 0):
        import numpy as np
        n = C.c_size_t()
        check(lib().tsn_dit_tap(self.h, name.encode(), arm, None, 0, C.byref(n)))
        out = np.empty(n.value, dtype=np.float32)
        check(lib().tsn_dit_tap(self.h, name.encode(), arm, out.ctypes.data, n.value, C.byref(n)))
        return out

    def step(self, t: float, cfg: float, dt: float):
        check(lib().tsn_dit_step(self.h, t, cfg, dt))

    def sample(self, steps: int, cfg: float):
        check(lib().tsn_dit_sample(self.h, steps, cfg))

    def schedule(self, steps: int, cfg: float):
        check(lib().tsn_dit_schedule(self.h, steps, cfg))

    def run_steps(self, n: int):
        check(lib().tsn_dit_run_steps(self.h, n))

    def split_schedule(self, steps: int):
        """CFG split (arms = 1): install the sampler's t / dt schedule and rewind it."""
        check(lib().tsn_dit_split_schedule(self.h, steps))

    def split_forward(self, flow_dev):
        """CFG split: issue this arm's forward at the schedule's step; flow [T, 64] f32 into flow_dev."""
        check(lib().tsn_dit_split_forward(self.h, _p(flow_dev)))

    def split_update(self, flows2_dev, cfg: float):
        """CFG split: x += dt (fu + cfg (fc - fu)) from flows2_dev [2, T, 64]; advance the schedule."""
        check(lib().tsn_dit_split_update(self.h, _p(flows2_dev), cfg))

    def step_host(self, x_in, x_out, t: float, cfg: float, dt: float):
        check(lib().tsn_dit_step_host(self.h, _p(x_in), _p(x_out), t, cfg, dt))

    def kernels_per_step(self) -> int:
        return lib().tsn_dit_kernels_per_step(self.h)

    def profile_step(self):
        out = (C.c_double * 5)()
        check(lib().tsn_dit_profile_step(self.h, out))
        return {"gemm_ms": out[0], "attn_ms": out[1], "other_ms": out[2], "gemm_flops": out[3],
                "gemm_launches": int(out[4])}


    def trace_op(self, op: int):
        """Per-CTA phase timestamps (ns) of stamped launch `op` (GEMM: 8 phases; adaLN, attention: 3): array [ctas, 8]."""
        import numpy as np
        n = C.c_int()
        out = np.zeros((4096, 8), np.uint64)
        check(lib().tsn_dit_trace_op(self.h, op, out.ctypes.data, 4096, C.byref(n)))
        return out[:min(n.value, 4096)]

    def timeline(self):
        """One eager forward with every GEMM, adaLN and attention launch stamped: array [launches, 5]
        of (op index, first entry, first work, last exit, median exit), ns from the forward's start."""
        import numpy as np
        n = C.c_int()
        out = np.zeros((8192, 5), np.float64)
        check(lib().tsn_dit_timeline(self.h, out.ctypes.data, 8192, C.byref(n)))
        return out[:min(n.value, 8192)]

    def autotune(self) -> str:
        buf = C.create_string_buffer(1 << 20)
        check(lib().tsn_dit_autotune(self.h, buf, len(buf)))
        return buf.value.decode()

    def tiles(self):
        """Tile of every GEMM launch: int32 array [gemms, 3] of (GEMM index, tile width, K slices)."""
        import numpy as np
        n = C.c_int()
        check(lib().tsn_dit_get_tiles(self.h, None, 0, C.byref(n)))
        out = np.zeros((max(n.value, 1), 3), np.int32)
        check(lib().tsn_dit_get_tiles(self.h, out.ctypes.data, n.value, C.byref(n)))
        return out[:n.value]

    def set_tiles(self, tiles) -> None:
        """Pin GEMM tiles (rows as `tiles()` returns them) and re-plan the forward."""
        import numpy as np
        t = np.ascontiguousarray(np.asarray(tiles, np.int32).reshape(-1, 3))
        check(lib().tsn_dit_set_tiles(self.h, t.ctypes.data, len(t)))

    def profile_ops(self) -> str:
        buf = C.create_string_buffer(1 << 20)
        check(lib().tsn_dit_profile_ops(self.h, buf, len(buf)))
        return buf.value.decode()


class TextEncoder:
    """tn::T5Model (kind "t5") or tn::ClipModel (kind "clip") on the device: 77 token ids ->
    per-token features [77, width] (and CLIP's pooled projection [width])."""

    def __init__(self, dev: Device, kind: str, gguf: str):
        if kind not in ("t5", "clip"):
            raise ValueError("kind must be 't5' or 'clip'")
        self.dev = dev
        self.kind = kind
        h = C.c_void_p()
        load = lib().tsn_t5_load if kind == "t5" else lib().tsn_clip_load
        check(load(dev.h, gguf.encode(), C.byref(h)))
        self.h = h
        w, n, layers = C.c_uint32(), C.c_uint32(), C.c_uint32()
        check(lib().tsn_encoder_info(h, C.byref(w), C.byref(n), C.byref(layers)))
        self.width, self.ctx, self.layers = w.value, n.value, layers.value
        dev._models.add(self)

    def encode(self, ids):
        """Host int32 ids [ctx] -> per_token [ctx, width] f32 (t5), or (per_token, pooled [width]) (clip)."""
        import numpy as np
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros((self.ctx, self.width), np.float32)
        pooled = np.zeros(self.width, np.float32)
        check(lib().tsn_encoder_encode(self.h, ids.ctypes.data, ids.size, out.ctypes.data, out.size,
                                       pooled.ctypes.data, pooled.size))
        return out if self.kind == "t5" else (out, pooled)

    def last_ms(self) -> float:
        return lib().tsn_encoder_last_ms(self.h)

    def flops(self) -> float:
        return lib().tsn_encoder_flops(self.h)

    def launches(self) -> int:
        """Kernel launches in one encode graph."""
        return lib().tsn_encoder_launches(self.h)

    def weight_bytes(self) -> float:
        return lib().tsn_encoder_weight_bytes(self.h)

    def profile_ops(self) -> str:
        buf = C.create_string_buffer(1 << 18)
        check(lib().tsn_encoder_profile_ops(self.h, buf, len(buf)))
        return buf.value.decode()

    def close(self):
        if self.h and self.dev.h:
            lib().tsn_encoder_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def write_synthetic_t5_gguf(path: str, d_model: int = 2048, d_ff: int = 5120, layers: int = 24, heads: int = 32,
                            seed: int = 4242):
    """The seeded synthetic T5 encoder GGUF (Q8_0 matrices; tensor names of src/t5.cpp)."""
    check(lib().tsn_gguf_write_synthetic_t5(path.encode(), d_model, d_ff, layers, heads, seed))


def write_synthetic_clip_gguf(path: str, hidden: int = 1024, layers: int = 24, heads: int = 16, seed: int = 4242):
    """The seeded synthetic MetaCLIP text encoder GGUF (f32; tensor names of src/clip.cpp)."""
    check(lib().tsn_gguf_write_synthetic_clip(path.encode(), hidden, layers, heads, seed))


def write_synthetic_vae_gguf(path: str, channels: int = 128, latent_dim: int = 64, out_channels: int = 2,
                             seed: int = 4242):
    """Seeded synthetic VAE decoder GGUF (f32; the tensor names src/vae.cpp reads)."""
    check(lib().tsn_gguf_write_synthetic_vae(path.encode(), latent_dim, channels, out_channels, seed))


def inspect(path: str):
    """Host-only check of a DiT GGUF (tsn_dit_inspect): (geometry, device weight bytes); raises
    TsnError with TSN_ERR_IO / FORMAT / MISSING / ARG. Needs no GPU."""
    g = Geom()
    nb = C.c_size_t()
    check(lib().tsn_dit_inspect(path.encode(), C.byref(g), C.byref(nb)))
    return g, nb.value


def write_synthetic_gguf(path: str, g: Geom, seed: int = 4242, with_prep: bool = False):
    check(lib().tsn_gguf_write_synthetic(path.encode(), C.byref(g), seed, int(with_prep)))
