"""ORACLE -- test infrastructure only (tests/, __graft_entry__.smoke, bench.py's
CPU-baseline leg).  Nothing in the product imports this module.

Two checkers live here:

1. `RefModel` / `ref_gemv_batch` / `ref_dequant_row`: ctypes bindings of the
   reference engine itself, compiled from its own sources by oracle/Makefile
   into oracle/_ref/libqwenref.so (see oracle/harness.c for the loop
   drivers).  This is the parity anchor: its outputs ARE the reference's.

2. `port_*`: a plain numpy restatement of the hot-path arithmetic, pinned
   against (1) by tests/test_oracle.py:
     port_dequant        <- src/quant.c:86-182 (Q8_0, Q4_K, Q5_K, Q6_K, IQ4_XS)
     port_gemv           <- src/kernels.c:323-599 (math, in float64)
     port_rmsnorm/l2norm <- src/kernels.c:741-805
     port_silu/sigmoid/softplus/softmax <- src/kernels.c:825-939
     port_gdn_step       <- src/model.c:494-524, 564-586
     port_argmax         <- src/model.c:746-756
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(_HERE, "_ref", "libqwenref.so")

KVALUES = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.int8)

_ref = None


def available():
    return os.path.exists(REF_LIB)


def ref():
    global _ref
    if _ref is None:
        if not available():
            raise RuntimeError(f"{REF_LIB} missing: build it with `make -C oracle` where the reference exists")
        L = C.CDLL(REF_LIB)
        vp, u32, i32, f32 = C.c_void_p, C.c_uint32, C.c_int, C.c_float
        P = C.POINTER
        L.ref_open.restype = vp
        L.ref_open.argtypes = [C.c_char_p, u32, i32]
        L.ref_close.argtypes = [vp]
        for n in ("ref_logits", "ref_logits_b", "ref_h_save", "ref_mtp_h", "ref_x", "ref_bx"):
            getattr(L, n).restype = P(f32)
            getattr(L, n).argtypes = [vp]
        for n in ("ref_get_pos", "ref_vocab", "ref_n_embd", "ref_n_layer"):
            getattr(L, n).restype = u32
            getattr(L, n).argtypes = [vp]
        L.ref_set_pos.argtypes = [vp, u32]
        L.ref_is_recurrent.argtypes = [vp, u32]
        L.ref_is_recurrent.restype = i32
        L.ref_layer_state.argtypes = [vp, u32, i32]
        L.ref_layer_state.restype = P(f32)
        L.ref_find_tensor.argtypes = [vp, C.c_char_p]
        L.ref_find_tensor.restype = vp
        L.ref_forward.argtypes = [vp, u32, u32]
        L.ref_forward_batch.argtypes = [vp, P(u32), u32, u32, i32]
        L.ref_rollback_to.argtypes = [vp, u32]
        L.ref_layer.argtypes = [vp, u32, u32]
        L.ref_mtp_forward.argtypes = [vp, u32, u32, i32]
        L.ref_mtp_forward_batch.argtypes = [vp, P(u32), u32, u32, i32]
        L.ref_argmax.argtypes = [P(f32), u32]
        L.ref_argmax.restype = u32
        L.ref_prefill.argtypes = [vp, P(u32), u32, i32]
        L.ref_spec_generate.argtypes = [vp, u32, u32, P(u32), u32, P(u32), P(u32), u32, P(u32)]
        L.ref_spec_generate.restype = u32
        L.ref_greedy_generate.argtypes = [vp, u32, P(u32)]
        L.ref_greedy_generate.restype = u32
        L.ref_make_tensor.argtypes = [vp, i32, C.c_uint64, C.c_uint64]
        L.ref_make_tensor.restype = vp
        L.ref_free_tensor.argtypes = [vp]
        L.ref_gemv_batch_any.argtypes = [vp, P(f32), C.c_uint64, i32, P(f32), C.c_uint64, i32]
        L.ref_gemv.argtypes = [vp, P(f32), P(f32), i32]
        L.dequant_row.argtypes = [i32, vp, C.c_uint64, P(f32)]
        L.dequant_row.restype = i32
        L.ref_spec_max_b.restype = i32
        L.sampler_init.argtypes = [f32, f32, u32, f32, C.c_uint64]
        L.sampler_init.restype = vp
        L.sampler_free.argtypes = [vp]
        L.sampler_sample.argtypes = [vp, P(f32), u32, P(u32), C.c_size_t]
        L.sampler_sample.restype = u32
        L.ref_sample_generate.argtypes = [vp, vp, u32, P(u32), u32, P(u32)]
        L.ref_sample_generate.restype = u32
        for n in ("rmsnorm",):
            getattr(L, n).argtypes = [P(f32), P(f32), P(f32), C.c_uint64, f32]
        L.l2norm.argtypes = [P(f32), P(f32), C.c_uint64, f32]
        for n in ("silu_inplace", "sigmoid_inplace", "softplus_inplace", "softmax_inplace"):
            getattr(L, n).argtypes = [P(f32), C.c_uint64]
        L.ref_now.restype = C.c_double
        _ref = L
    return _ref


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _up(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


# ------------------------------ reference engine ------------------------------

class RefModel:
    """The reference qwen_model_t + a thread pool (oracle/harness.c)."""

    def __init__(self, path, n_ctx, n_threads=0):
        self.h = ref().ref_open(os.fsencode(path), n_ctx, n_threads)
        if not self.h:
            raise RuntimeError(f"reference model_init failed for {path}")
        self.V = ref().ref_vocab(self.h)
        self.E = ref().ref_n_embd(self.h)
        self.n_layer = ref().ref_n_layer(self.h)

    def close(self):
        if self.h:
            ref().ref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self):
        return ref().ref_get_pos(self.h)

    @pos.setter
    def pos(self, v):
        ref().ref_set_pos(self.h, v)

    def logits(self):
        return np.ctypeslib.as_array(ref().ref_logits(self.h), (self.V,)).copy()

    def logits_b(self, B):
        return np.ctypeslib.as_array(ref().ref_logits_b(self.h), (B * self.V,)).reshape(B, self.V).copy()

    def h_save(self, B):
        return np.ctypeslib.as_array(ref().ref_h_save(self.h), (B * self.E,)).reshape(B, self.E).copy()

    def mtp_h(self):
        return np.ctypeslib.as_array(ref().ref_mtp_h(self.h), (self.E,))

    def x(self):
        return np.ctypeslib.as_array(ref().ref_x(self.h), (self.E,)).copy()

    def is_recurrent(self, il):
        return bool(ref().ref_is_recurrent(self.h, il))

    def state(self, il, which, n):
        p = ref().ref_layer_state(self.h, il, which)
        return np.ctypeslib.as_array(p, (n,)).copy()

    def set_x(self, v):
        np.ctypeslib.as_array(ref().ref_x(self.h), (self.E,))[:] = v

    def layer(self, il, pos):
        ref().ref_layer(self.h, il, pos)

    def forward(self, tok, pos):
        ref().ref_forward(self.h, tok, pos)

    def forward_batch(self, toks, pos, ckpt):
        t = np.ascontiguousarray(toks, np.uint32)
        ref().ref_forward_batch(self.h, _up(t), pos, t.size, ckpt)

    def rollback_to(self, b):
        ref().ref_rollback_to(self.h, b)

    def mtp_forward(self, tok, pos, want):
        ref().ref_mtp_forward(self.h, tok, pos, want)

    def mtp_forward_batch(self, toks, pos, want):
        t = np.ascontiguousarray(toks, np.uint32)
        ref().ref_mtp_forward_batch(self.h, _up(t), pos, t.size, want)

    def prefill(self, toks, spec):
        t = np.ascontiguousarray(toks, np.uint32)
        ref().ref_prefill(self.h, _up(t), t.size, spec)

    def spec_generate(self, n_predict, n_spec=3, forced=None, max_cycles=100000):
        out = np.zeros(n_predict + 8, np.uint32)
        js = np.zeros(max_cycles, np.uint32)
        nc = C.c_uint32()
        f = np.ascontiguousarray(forced if forced is not None else [], np.uint32)
        n = ref().ref_spec_generate(self.h, n_predict, n_spec, _up(f) if f.size else None, f.size, _up(out),
                                    _up(js), max_cycles, C.byref(nc))
        return out[:n].copy(), js[:nc.value].copy()

    def sample_generate(self, sampler, n_predict, history):
        """src/main.c:232-248 with the reference sampler (RefSampler)."""
        h = np.zeros(len(history) + n_predict + 1, np.uint32)
        h[:len(history)] = history
        out = np.zeros(n_predict + 1, np.uint32)
        n = ref().ref_sample_generate(self.h, sampler.s, n_predict, _up(h), len(history), _up(out))
        return out[:n].copy()

    def greedy_generate(self, n_predict):
        out = np.zeros(n_predict + 1, np.uint32)
        n = ref().ref_greedy_generate(self.h, n_predict, _up(out))
        return out[:n].copy()


class RefSampler:
    """The reference sampler (src/sampler.c) itself, from oracle/_ref."""

    def __init__(self, temp, top_p, top_k, repeat_penalty, seed):
        self.s = ref().sampler_init(temp, top_p, top_k, repeat_penalty, seed)

    @property
    def rng_state(self):
        # sampler_t: float, float, u32, float, u32, (pad), u64
        return C.c_uint64.from_address(self.s + 24).value

    def sample(self, logits, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        return ref().sampler_sample(self.s, _fp(logits), logits.size, _up(t) if t.size else None, t.size)

    def close(self):
        if self.s:
            ref().sampler_free(self.s)
            self.s = None


def ref_gemv_batch(data, gtype, ne0, ne1, x, n_threads=0):
    """Reference gemv_batch (src/kernels.c:640-648) for any n (chunks of 8)."""
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[0]
    out = np.zeros((n, ne1), np.float32)
    t = ref().ref_make_tensor(data.ctypes.data, gtype, ne0, ne1)
    try:
        ref().ref_gemv_batch_any(t, _fp(x), x.shape[1], n, _fp(out), ne1, n_threads)
    finally:
        ref().ref_free_tensor(t)
    return out


def ref_gemv(data, gtype, ne0, ne1, x, n_threads=0):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(ne1, np.float32)
    t = ref().ref_make_tensor(data.ctypes.data, gtype, ne0, ne1)
    try:
        ref().ref_gemv(t, _fp(x), _fp(out), n_threads)
    finally:
        ref().ref_free_tensor(t)
    return out


def ref_dequant_row(data, gtype, ne0):
    out = np.zeros(ne0, np.float32)
    if ref().dequant_row(gtype, data.ctypes.data, ne0, _fp(out)) != 0:
        raise ValueError("dequant_row rejected the format")
    return out


def ref_op(name, x, w=None, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32).copy()
    L = ref()
    if name == "rmsnorm":
        out = np.empty_like(x)
        L.rmsnorm(_fp(out), _fp(x), _fp(np.ascontiguousarray(w, np.float32)) if w is not None else None, x.size, eps)
        return out
    if name == "l2norm":
        out = np.empty_like(x)
        L.l2norm(_fp(out), _fp(x), x.size, eps)
        return out
    getattr(L, name + "_inplace")(_fp(x), x.size)
    return x


# --------------------------------- numpy port ----------------------------------

def _f16(u16):
    return u16.view(np.float16).astype(np.float32)


def port_dequant(raw, gtype, ne0):
    """Dequantise rows of GGUF blocks: raw uint8 [rows * row_bytes] -> float32 [rows, ne0]."""
    raw = np.asarray(raw, np.uint8)
    if gtype == 0:
        return raw.view(np.float32).reshape(-1, ne0)
    if gtype == 8:    # Q8_0: d(f16) qs[32]  (src/quant.c:86-92)
        b = raw.reshape(-1, 34)
        d = _f16(b[:, :2].copy().view(np.uint16)[:, 0])
        q = b[:, 2:].view(np.int8).astype(np.float32)
        return (d[:, None] * q).reshape(-1, ne0)
    if gtype == 23:   # IQ4_XS (src/quant.c:166-182)
        b = raw.reshape(-1, 136)
        d = _f16(b[:, :2].copy().view(np.uint16)[:, 0])
        sh = b[:, 2:4].copy().view(np.uint16)[:, 0].astype(np.int32)
        sl = b[:, 4:8].astype(np.int32)
        qs = b[:, 8:].reshape(-1, 8, 16).astype(np.int32)
        ib = np.arange(8)
        ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh[:, None] >> (2 * ib)) & 3) << 4)
        dl = (d[:, None] * (ls - 32).astype(np.float32)).astype(np.float32)
        lo = KVALUES[qs & 0xF].astype(np.float32)
        hi = KVALUES[qs >> 4].astype(np.float32)
        y = np.concatenate([dl[:, :, None] * lo, dl[:, :, None] * hi], axis=2)
        return y.astype(np.float32).reshape(-1, ne0)
    if gtype == 14:   # Q6_K (src/quant.c:140-164)
        b = raw.reshape(-1, 210)
        ql = b[:, :128].astype(np.int32)
        qh = b[:, 128:192].astype(np.int32)
        sc = b[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(b[:, 208:210].copy().view(np.uint16)[:, 0])
        y = np.zeros((b.shape[0], 256), np.float32)
        for n in range(2):
            for l in range(32):
                isx = l // 16
                f = np.float32
                q1 = (((ql[:, 64 * n + l] & 0xF) | (((qh[:, 32 * n + l] >> 0) & 3) << 4)) - 32).astype(f)
                q2 = (((ql[:, 64 * n + l + 32] & 0xF) | (((qh[:, 32 * n + l] >> 2) & 3) << 4)) - 32).astype(f)
                q3 = (((ql[:, 64 * n + l] >> 4) | (((qh[:, 32 * n + l] >> 4) & 3) << 4)) - 32).astype(f)
                q4 = (((ql[:, 64 * n + l + 32] >> 4) | (((qh[:, 32 * n + l] >> 6) & 3) << 4)) - 32).astype(f)
                base = 128 * n
                y[:, base + l] = (d * sc[:, 8 * n + isx]) * q1
                y[:, base + l + 32] = (d * sc[:, 8 * n + isx + 2]) * q2
                y[:, base + l + 64] = (d * sc[:, 8 * n + isx + 4]) * q3
                y[:, base + l + 96] = (d * sc[:, 8 * n + isx + 6]) * q4
        return y.reshape(-1, ne0)
    if gtype in (12, 13):  # Q4_K / Q5_K (src/quant.c:94-138; include/quant.h:21-29)
        bb = 144 if gtype == 12 else 176
        b = raw.reshape(-1, bb)
        d = _f16(b[:, :2].copy().view(np.uint16)[:, 0])
        dm = _f16(b[:, 2:4].copy().view(np.uint16)[:, 0])
        s = b[:, 4:16].astype(np.int32)
        qh = b[:, 16:48].astype(np.int32) if gtype == 13 else None
        qs = b[:, 48:].astype(np.int32) if gtype == 13 else b[:, 16:].astype(np.int32)
        y = np.zeros((b.shape[0], 256), np.float32)
        for j in range(8):
            if j < 4:
                sc, m = s[:, j] & 63, s[:, j + 4] & 63
            else:
                sc = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
                m = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
            d1 = (d * sc.astype(np.float32)).astype(np.float32)
            m1 = (dm * m.astype(np.float32)).astype(np.float32)
            q = qs[:, 32 * (j // 2):32 * (j // 2) + 32]
            q = (q & 0xF) if j % 2 == 0 else (q >> 4)
            if qh is not None:
                q = q + np.where((qh >> j) & 1, 16, 0)
            y[:, 32 * j:32 * j + 32] = (d1[:, None] * q.astype(np.float32)) - m1[:, None]
        return y.reshape(-1, ne0)
    raise ValueError(f"type {gtype}")


def port_gemv(raw, gtype, ne0, x):
    """out[t][r] = sum_k W[r][k] x[t][k] in float64 (the reference's math)."""
    W = port_dequant(raw, gtype, ne0).astype(np.float64)
    return np.asarray(x, np.float64) @ W.T


def port_rmsnorm(x, w, eps):
    x = np.asarray(x, np.float64)
    s = 1.0 / np.sqrt(np.mean(x * x) + eps)
    return x * s * (np.asarray(w, np.float64) if w is not None else 1.0)


def port_l2norm(x, eps):
    x = np.asarray(x, np.float64)
    return x / max(np.sqrt(np.sum(x * x)), eps)


def port_silu(x):
    x = np.asarray(x, np.float64)
    return x / (1.0 + np.exp(-x))


def port_sigmoid(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def port_softplus(x):
    x = np.asarray(x, np.float64)
    return np.where(x > 30.0, x, np.log1p(np.exp(np.minimum(x, 30.0))))


def port_softmax(x):
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max())
    return e / e.sum()


def port_gdn_step(S, q, k, v, beta_raw, alpha_raw, dt_bias, ssm_a):
    """One token of one v-head (src/model.c:494-524, 572-586), float64.
    S: [dv][dk] state, q/k L2-normalised.  Returns (S', out)."""
    S = np.asarray(S, np.float64)
    b = 1.0 / (1.0 + np.exp(-beta_raw))
    a = alpha_raw + dt_bias
    sp = a if a > 30.0 else np.log1p(np.exp(a))
    decay = np.exp(ssm_a * sp)
    kq = float(np.dot(k, q))
    sk = S @ k
    sq = S @ q
    dj = (v - decay * sk) * b
    out = (decay * sq + dj * kq) / np.sqrt(len(k))
    S2 = decay * S + np.outer(dj, k)
    return S2, out


def port_argmax(x):
    """The scan of src/model.c:746-756: max seeded with x[0], replaced only when
    x[i] > max.  So the first maximum wins, -0 equals +0, a NaN never wins,
    and a NaN at x[0] makes every comparison false (result 0)."""
    x = np.asarray(x, np.float32)
    if np.isnan(x[0]):
        return 0
    m = np.nanmax(x)
    return int(np.flatnonzero(x == m)[0])
