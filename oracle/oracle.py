"""Python access to the CPU oracle (TEST INFRASTRUCTURE — the parity checker).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may use this
module. It wraps:
  * lib/liboracle.so  — the CPU restatement of the reference's DiT path (port.cpp + kernels.cpp)
  * _ref/ts_ref_dit   — the reference's own host code (src/dit.cpp, src/dit_fwd.cpp, src/net.mm,
                        src/gguf.cpp) built over a CPU Device; present only where it was built.
  * _ref/ts_ref_dit_tsn — the same host code and driver over the GPU through the library's drop-in
                        device (integration/gpu_tsn.cpp): the tests check the boundary with it.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "lib", "liboracle.so")
REF_BIN = os.path.join(HERE, "_ref", "ts_ref_dit")
REF_TSN_BIN = os.path.join(HERE, "_ref", "ts_ref_dit_tsn")

TAPS = ["t_emb", "global_c", "extended_c", "x_in", "text_xn", "a0_q", "a0_k", "a0_v", "a0_out",
        "jb0_lat", "jb0_clip", "jb0_text", "after_joint", "after_fused", "final_fx", "final_mod", "flow"]

_F = C.POINTER(C.c_float)


def _f(a):
    return a.ctypes.data_as(_F) if a is not None else None


class Oracle:
    def __init__(self, gguf: str):
        self.L = C.CDLL(LIB)
        L = self.L
        L.oracle_load.restype = C.c_void_p
        L.oracle_load.argtypes = [C.c_char_p]
        L.oracle_free.argtypes = [C.c_void_p]
        L.oracle_info.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        L.oracle_threads.restype = C.c_int
        L.oracle_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _F, C.c_float, _F, _F, _F, _F, _F, C.c_int]
        L.oracle_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _F, C.c_float, C.c_float, C.c_float,
                                  _F, _F, _F, _F, _F, _F, _F, _F]
        L.oracle_prep.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int] + [_F] * 12
        L.oracle_joint_block.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _F, _F, _F, _F, _F]
        L.oracle_tap.restype = C.c_longlong
        L.oracle_tap.argtypes = [C.c_void_p, C.c_char_p, _F, C.c_longlong]
        self.h = L.oracle_load(gguf.encode())
        if not self.h:
            raise RuntimeError(f"oracle could not load {gguf}")
        info = (C.c_int * 6)()
        L.oracle_info(self.h, info)
        self.H, self.NH, self.F, self.depth, self.fused_depth, self.latent_dim = list(info)

    def close(self):
        if self.h:
            self.L.oracle_free(self.h)
            self.h = None

    def threads(self) -> int:
        return self.L.oracle_threads()

    def forward(self, T, C_, TS, x, t, clip_pp, sync_gather, text_pp, gcmlp, taps=False):
        flow = np.zeros((T, self.latent_dim), np.float32)
        args = [np.ascontiguousarray(a, dtype=np.float32) for a in (x, clip_pp, sync_gather, text_pp, gcmlp)]
        self.L.oracle_forward(self.h, T, C_, TS, _f(args[0]), t, _f(args[1]), _f(args[2]), _f(args[3]),
                              _f(args[4]), _f(flow), int(taps))
        return flow

    def joint_block(self, lat, clip, text, extc_silu, global_c_silu):
        """Joint block 0 (src/dit_fwd.cpp:180-257) for one arm; returns the updated (lat, clip, text)."""
        T, C_, TS = lat.shape[0], clip.shape[0], text.shape[0]
        lat, clip, text = (np.array(v, np.float32, copy=True) for v in (lat, clip, text))
        e, g = (np.ascontiguousarray(v, dtype=np.float32) for v in (extc_silu, global_c_silu))
        if self.L.oracle_joint_block(self.h, T, C_, TS, _f(lat), _f(clip), _f(text), _f(e), _f(g)) != 0:
            raise RuntimeError("oracle_joint_block needs two or more joint blocks")
        return lat, clip, text

    def tap(self, name: str) -> np.ndarray:
        n = self.L.oracle_tap(self.h, name.encode(), None, 0)
        if n < 0:
            raise KeyError(name)
        out = np.empty(n, np.float32)
        self.L.oracle_tap(self.h, name.encode(), _f(out), n)
        return out

    def step(self, T, C_, TS, x, t, cfg, dt, clip_pp, sync_gather, tp_c, gc_c, tp_u, gc_u):
        x = np.array(x, np.float32, copy=True)
        fc = np.zeros_like(x)
        fu = np.zeros_like(x)
        a = [np.ascontiguousarray(v, dtype=np.float32) for v in (clip_pp, sync_gather, tp_c, gc_c, tp_u, gc_u)]
        self.L.oracle_step(self.h, T, C_, TS, _f(x), t, cfg, dt, *[_f(v) for v in a], _f(fc), _f(fu))
        return x, fc, fu

    def prep(self, T, C_, TS, sync_S, clip_f, sync_f, text_cat_c, gtext_c, text_cat_u, gtext_u):
        """prep_conditioning + prep_text_arm (src/dit.cpp:55-192) for both arms; needs H = 1024.
        Returns a dict of PREP_OUT arrays."""
        H = self.H
        out = {"clip_pp": np.zeros((C_, H), np.float32), "sync_gather": np.zeros((T, H), np.float32),
               "text_pp_cond": np.zeros((TS, H), np.float32), "gcmlp_cond": np.zeros(H, np.float32),
               "text_pp_unc": np.zeros((TS, H), np.float32), "gcmlp_unc": np.zeros(H, np.float32)}
        a = [np.ascontiguousarray(v, dtype=np.float32) for v in (clip_f, sync_f, text_cat_c, gtext_c, text_cat_u, gtext_u)]
        rc = self.L.oracle_prep(self.h, T, C_, TS, sync_S, *[_f(v) for v in a], *[_f(out[k]) for k in PREP_OUT])
        if rc != 0:
            raise RuntimeError("oracle_prep needs a model with H = 1024")
        return out


PREP_OUT = ("clip_pp", "sync_gather", "text_pp_cond", "gcmlp_cond", "text_pp_unc", "gcmlp_unc")


def write_synthetic_gguf(path: str, H=1024, NH=16, F=4096, depth=21, fused_depth=14, latent_dim=64,
                         rope_theta=10000.0, t_max_period=1.0, seed=4242, with_prep=False):
    """The seeded synthetic DiT GGUF (byte-identical to tsn.write_synthetic_gguf), written by
    liboracle.so so that a CPU-only process never loads the GPU library."""
    L = C.CDLL(LIB)
    L.oracle_write_synthetic_gguf.restype = C.c_int
    L.oracle_write_synthetic_gguf.argtypes = [C.c_char_p] + [C.c_uint] * 6 + [C.c_float, C.c_float, C.c_ulonglong,
                                                                              C.c_int]
    if L.oracle_write_synthetic_gguf(path.encode(), H, NH, F, depth, fused_depth, latent_dim, rope_theta, t_max_period,
                                     seed, int(with_prep)) != 0:
        raise RuntimeError(f"could not write {path}")


def have_ref() -> bool:
    return os.access(REF_BIN, os.X_OK)


def write_inputs(d: str, inputs: dict):
    os.makedirs(d, exist_ok=True)
    for k, v in inputs.items():
        np.ascontiguousarray(v, dtype=np.float32).tofile(os.path.join(d, f"{k}.bin"))


def run_ref(mode: str, gguf: str, T: int, C_: int, TS: int, in_dir: str, out_dir: str, *args, threads=None,
            timeout=3600, binary=None):
    """Run the reference-built driver (binary: REF_TSN_BIN for its GPU build); returns its stdout."""
    os.makedirs(out_dir, exist_ok=True)
    env = dict(os.environ)
    if threads:
        env["OMP_NUM_THREADS"] = str(threads)
    cmd = [binary or REF_BIN, mode, gguf, str(T), str(C_), str(TS), in_dir, out_dir] + [str(a) for a in args]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"ts_ref_dit failed ({r.returncode}): {r.stderr[-2000:]}")
    return r.stdout


def read_ref_taps(out_dir: str) -> dict:
    taps = {}
    for name in TAPS:
        p = os.path.join(out_dir, f"nat_{name}.bin") if name != "flow" else os.path.join(out_dir, "flow.bin")
        if os.path.exists(p):
            taps[name] = np.fromfile(p, np.float32)
    return taps


def parse_json_line(s: str) -> dict:
    for line in s.splitlines()[::-1]:
        line = line.strip()
        if line.startswith("{"):
            return json.loads(line)
    raise ValueError("no JSON line in output")


# ---------------------------------------------------------------- VAE decoder (src/vae.cpp)
VAE_STRIDES = (8, 8, 4, 4, 2)
VAE_DILS = (1, 3, 9)


def ref_vae(gguf: str, latent: np.ndarray, threads=None, reps=1, workdir=None, binary=None):
    """VaeModel::decode of the reference build (src/vae.cpp:17-86) on latent [T, 64].
    Returns (audio [T_audio, 2] f32, timing JSON)."""
    import tempfile
    d = workdir or tempfile.mkdtemp(prefix="tsn_vae_")
    write_inputs(d, {"latent": latent})
    out = run_ref("vae", gguf, latent.shape[0], 0, 0, d, d, reps, threads=threads, binary=binary)
    js = parse_json_line(out)
    audio = np.fromfile(os.path.join(d, "audio.bin"), np.float32).reshape(-1, 2)
    return audio, js


def _conv1d_np(x, w, b, stride=1, pad=0, dil=1, convt=False, OL=None):
    """conv1d as the reference's im2col + GEMM (shaders/ops_conv.metal:262-283): x [T, IC],
    w [OC, IC, K]; with convt the input is zero-stuffed by `stride` and convolved at stride 1."""
    T, IC = x.shape
    OC, _, K = w.shape
    OL = T if OL is None else OL
    t = np.arange(OL)[:, None]
    k = np.arange(K)[None, :]
    if convt:
        ui = t - pad + k
        ok = (ui >= 0) & (ui % stride == 0)
        ti = ui // stride
    else:
        ti = t * stride - pad + k * dil
        ok = np.ones_like(ti, dtype=bool)
    ok = ok & (ti >= 0) & (ti < T)
    col = np.where(ok[:, :, None], x[np.clip(ti, 0, T - 1)], 0.0)   # [OL, K, IC]
    y = np.einsum("tki,oik->to", col, w, optimize=True)
    return y + b if b is not None else y


def _snake_np(x, alpha, beta):
    """snake_ (shaders/ops_conv.metal:204-213): x + sin(x e^alpha)^2 e^-beta, per channel."""
    s = np.sin(x * np.exp(alpha))
    return x + s * s * np.exp(-beta)


def vae_decode_np(W, latent):
    """Float64 restatement of VaeModel::decode (src/vae.cpp:17-86) for small cases.
    W(name) returns a tensor as numpy: conv weights [OC, IC, K], vectors [n]."""
    x = _conv1d_np(latent.astype(np.float64), W("decoder.layers.0.weight"), W("decoder.layers.0.bias"), pad=3)
    for n, st in enumerate(VAE_STRIDES):
        bp = f"decoder.layers.{n + 1}"
        h = _snake_np(x, W(bp + ".layers.0.alpha"), W(bp + ".layers.0.beta"))
        w = W(bp + ".layers.1.weight")
        K = w.shape[2]
        x = _conv1d_np(h, w, W(bp + ".layers.1.bias"), stride=st, pad=K - 1 - st // 2, convt=True, OL=h.shape[0] * st)
        for r, dl in enumerate(VAE_DILS):
            rp = f"{bp}.layers.{r + 2}"
            h = _snake_np(x, W(rp + ".layers.0.alpha"), W(rp + ".layers.0.beta"))
            g = _conv1d_np(h, W(rp + ".layers.1.weight"), W(rp + ".layers.1.bias"), pad=3 * dl, dil=dl)
            h = _snake_np(g, W(rp + ".layers.2.alpha"), W(rp + ".layers.2.beta"))
            x = x + _conv1d_np(h, W(rp + ".layers.3.weight"), W(rp + ".layers.3.bias"))
    h = _snake_np(x, W("decoder.layers.6.alpha"), W("decoder.layers.6.beta"))
    return _conv1d_np(h, W("decoder.layers.7.weight"), None, pad=3)



# ------------------------------------------------ text encoders (src/t5.cpp, src/clip.cpp)
def ref_encoder(kind: str, gguf: str, ids: np.ndarray, threads=None, reps=1, workdir=None, binary=None):
    """T5Model::encode (kind "t5", src/t5.cpp:84-131) or ClipModel::encode ("clip",
    src/clip.cpp:30-101) of the reference build on 77 int32 ids. Returns (per_token [77, width],
    pooled [width] or None, timing JSON)."""
    import tempfile
    d = workdir or tempfile.mkdtemp(prefix="tsn_enc_")
    os.makedirs(d, exist_ok=True)
    np.ascontiguousarray(ids, np.int32).tofile(os.path.join(d, "ids.bin"))
    js = parse_json_line(run_ref(kind, gguf, 0, 0, 0, d, d, reps, threads=threads, binary=binary))
    if kind == "t5":
        return np.fromfile(os.path.join(d, "out.bin"), np.float32).reshape(77, -1), None, js
    pt = np.fromfile(os.path.join(d, "per_token.bin"), np.float32)
    g = np.fromfile(os.path.join(d, "global.bin"), np.float32)
    return pt.reshape(-1, g.size), g, js


def t5_bucket(rel: int, num_buckets: int, max_dist: int) -> int:
    """T5's bidirectional relative-position bucket (src/t5.cpp:7-20)."""
    ret = 0
    num_buckets //= 2
    if rel > 0:
        ret += num_buckets
    n = abs(rel)
    max_exact = num_buckets // 2
    if n < max_exact:
        return ret + n
    v = max_exact + int(np.log(n / max_exact) / np.log(max_dist / max_exact) * (num_buckets - max_exact))
    return ret + min(v, num_buckets - 1)


def _softmax_rows(s):
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / e.sum(axis=-1, keepdims=True)


def _heads_attention(q, k, v, nh, scale, bias):
    """softmax(scale q kᵀ + bias) v per head (attn_qk / softmax_rows / attn_pav,
    shaders/gemm_attn.metal:96-202); bias [nh, n, n] with -inf for masked keys."""
    n, d = q.shape
    hd = d // nh
    out = np.zeros_like(q)
    for h in range(nh):
        sl = slice(h * hd, (h + 1) * hd)
        s = scale * (q[:, sl] @ k[:, sl].T) + bias[h]
        out[:, sl] = _softmax_rows(s) @ v[:, sl]
    return out


def t5_encode_np(W, kv: dict, ids: np.ndarray) -> np.ndarray:
    """Float64 restatement of T5Model::encode (src/t5.cpp:84-131). W(name) gives a tensor as the
    reference's device holds it (matrices [N, K], vectors [n]), W(name, host=True) the to_f32 values
    of its host copies (the embedding table); kv the GGUF's t5.* keys."""
    d, nh, L = kv["t5.d_model"], kv["t5.n_heads"], kv["t5.n_layers"]
    nb, md = kv.get("t5.rel_buckets", 32), kv.get("t5.rel_max_dist", 128)
    eps = kv.get("t5.eps", 1e-6)
    n = ids.size
    x = W("tok_emb", host=True).reshape(-1, d)[ids].astype(np.float64)   # host gather of to_f32 values
    rb = W("rel_bias").reshape(nb, nh)
    bk = np.array([[t5_bucket(k - q, nb, md) for k in range(n)] for q in range(n)])
    bias = np.transpose(rb[bk], (2, 0, 1)).copy()             # [nh, q, k]
    bias[:, :, ids == 0] = -np.inf                           # pad keys (pad_on)

    def rms(v, w):
        return v / np.sqrt((v * v).mean(axis=1, keepdims=True) + eps) * w

    def gelu_tanh(a):
        arg = 0.7978845608 * (a + 0.044715 * a ** 3)
        return 0.5 * a * (1.0 + np.tanh(np.clip(arg, -10.0, 10.0)))

    for l in range(L):
        bp = f"blk.{l}"
        r = rms(x, W(bp + ".attn_norm"))
        q, k, v = r @ W(bp + ".q").T, r @ W(bp + ".k").T, r @ W(bp + ".v").T
        x = x + _heads_attention(q, k, v, nh, 1.0, bias) @ W(bp + ".o").T
        r = rms(x, W(bp + ".ffn_norm"))
        x = x + (gelu_tanh(r @ W(bp + ".wi_0").T) * (r @ W(bp + ".wi_1").T)) @ W(bp + ".wo").T
    return rms(x, W("out_norm"))


def clip_encode_np(W, kv: dict, ids: np.ndarray):
    """Float64 restatement of ClipModel::encode (src/clip.cpp:30-101): (per_token [n, H], pooled [H])."""
    H, nh, L = kv["clip.hidden"], kv["clip.heads"], kv["clip.layers"]
    n = ids.size
    x = W("tok_emb", host=True).reshape(-1, H)[ids] + W("pos_emb", host=True).reshape(-1, H)[:n]
    eot = int(np.argmax(ids))                                 # first position of the largest id
    q_i, k_i = np.meshgrid(np.arange(n), np.arange(n), indexing="ij")
    bias = np.where((k_i <= q_i) & (k_i <= eot), 0.0, -np.inf)[None].repeat(nh, axis=0)

    def ln(v, w, b):
        m = v.mean(axis=1, keepdims=True)
        var = ((v - m) ** 2).mean(axis=1, keepdims=True)
        return (v - m) / np.sqrt(var + 1e-5) * w + b

    for l in range(L):
        bp = f"blk.{l}"
        r = ln(x, W(bp + ".ln1.w"), W(bp + ".ln1.b"))
        q = r @ W(bp + ".q.w").T + W(bp + ".q.b")
        k = r @ W(bp + ".k.w").T + W(bp + ".k.b")
        v = r @ W(bp + ".v.w").T + W(bp + ".v.b")
        a = _heads_attention(q, k, v, nh, 1.0 / np.sqrt(H // nh), bias)
        x = x + a @ W(bp + ".out.w").T + W(bp + ".out.b")
        r = ln(x, W(bp + ".ln2.w"), W(bp + ".ln2.b"))
        hdn = r @ W(bp + ".fc1.w").T + W(bp + ".fc1.b")
        hdn = hdn / (1.0 + np.exp(-1.702 * hdn))
        x = x + hdn @ W(bp + ".fc2.w").T + W(bp + ".fc2.b")
    pt = ln(x, W("out_ln.w"), W("out_ln.b"))
    return pt, W("text_proj").reshape(H, H) @ pt[eot]
