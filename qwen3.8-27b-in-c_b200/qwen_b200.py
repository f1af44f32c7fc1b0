"""Python host-side mirror of libqwenb200 (include/qwen_b200.h).

The functions keep the reference names and argument meaning
(include/model.h:117-148, include/kernels.h:11-44) with numpy arrays in
place of raw pointers, so the parity tests read like the reference's own
tests.  Everything computes on the GPU through the C ABI; loading fails
loudly when the CUDA library is missing.
"""
import ctypes as C
import os

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("QB_LIB", os.path.join(_PKG, "libqwenb200.so"))
SYNTH_PATH = os.path.join(_PKG, "libqbsynth.so")

GGML_F32, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_IQ4_XS = 0, 8, 12, 13, 14, 23
BLOCK = {GGML_F32: (1, 4), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144), GGML_Q5_K: (256, 176),
         GGML_Q6_K: (256, 210), GGML_IQ4_XS: (256, 136)}

# symbols declared in include/qwen_b200.h (checked by the CPU test suite)
EXPORTED = [
    "pool_create", "pool_destroy", "pool_run",
    "model_init", "model_free", "attention_layer", "gdn_layer", "model_forward", "model_forward_batch",
    "model_snapshot_states",
    "model_rollback_states", "model_rollback_to", "mtp_forward", "mtp_forward_batch",
    "model_sample_greedy",
    "gemv_rows", "gemv", "gemv_rows_batch", "gemv_batch", "gemv_multi", "gemv_multi_batch",
    "rmsnorm", "l2norm", "silu_inplace", "sigmoid_inplace", "softplus_inplace", "softmax_inplace",
    "qb_last_error", "qb_last_error_str", "qb_clear_error", "qb_prefill", "qb_spec_generate",
    "qb_greedy_generate", "qb_last_argmax", "qb_last_loop_ms", "qb_read_state", "qb_read_buffer",
    "qb_reset", "qb_bench", "qb_model_init_tp", "qb_tp_handle", "qb_tp_connect", "qb_tp_rows",
    "qb_argmax_rows_noalloc", "sampler_init", "sampler_free", "sampler_sample", "qb_sample_generate",
    "qb_seq_init", "qb_seq_prefill", "qb_seq_generate", "qb_enable_wide",
]


def row_bytes(gtype, ne0):
    be, bb = BLOCK[gtype]
    return ne0 // be * bb


class TensorInfo(C.Structure):
    """gguf_tensor_info_t (reference include/gguf.h:66-73)."""
    _fields_ = [("name", C.c_char * 64), ("n_dims", C.c_uint32), ("ne", C.c_uint64 * 4),
                ("type", C.c_int), ("offset", C.c_uint64), ("data", C.c_void_p)]


class QwenConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_embd", "n_head", "n_head_kv", "head_dim", "n_layer", "n_ff",
                                           "vocab_size", "context_len")] + [
        ("rope_theta", C.c_float), ("rope_dim_count", C.c_uint32), ("rope_sections", C.c_uint32 * 4),
        ("rms_norm_eps", C.c_float), ("tie_word_embeddings", C.c_bool)] + [
        (n, C.c_uint32) for n in ("full_attn_interval", "ssm_state_size", "ssm_conv_kernel",
                                  "ssm_inner_size", "ssm_group_count", "nextn_layers")]


class QwenDims(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_embd", "n_ff", "n_layer", "n_attn_layer", "n_recr_layer",
                                           "n_head", "n_kv_head", "head_dim")] + [
        ("rope_sections", C.c_uint32 * 4)] + [
        (n, C.c_uint32) for n in ("n_v_heads", "n_k_heads", "head_k_dim", "head_v_dim", "d_inner",
                                  "conv_dim", "d_conv", "d_state")]


class QwenLayer(C.Structure):
    _fields_ = [("index", C.c_uint32), ("is_recurrent", C.c_bool)]


class QwenModel(C.Structure):
    _fields_ = [("cfg", QwenConfig), ("dims", QwenDims), ("mtp_h", C.POINTER(C.c_float)),
                ("x", C.POINTER(C.c_float)), ("logits", C.POINTER(C.c_float)),
                ("logits_b", C.POINTER(C.c_float)), ("h_save", C.POINTER(C.c_float)),
                ("n_ctx", C.c_uint32), ("pos", C.c_uint32), ("layers", C.POINTER(QwenLayer)),
                ("eng", C.c_void_p)]


class SamplerT(C.Structure):
    """sampler_t (reference include/sampler.h:7-14)."""
    _fields_ = [("temp", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32), ("repeat_penalty", C.c_float),
                ("repeat_last_n", C.c_uint32), ("rng_state", C.c_uint64)]


_lib = None


def lib():
    """Load libqwenb200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run qwen3.8-27b-in-c_b200/build.py")
        L = C.CDLL(LIB_PATH)
        u32, i32, f32, vp = C.c_uint32, C.c_int, C.c_float, C.c_void_p
        P = C.POINTER
        L.model_init.argtypes = [P(QwenModel), C.c_char_p, u32]
        L.model_init.restype = i32
        L.model_free.argtypes = [P(QwenModel)]
        L.model_forward.argtypes = [P(QwenModel), vp, u32, u32]
        L.attention_layer.argtypes = [P(QwenModel), P(QwenLayer), vp, u32]
        L.gdn_layer.argtypes = [P(QwenModel), P(QwenLayer), vp]
        L.model_forward_batch.argtypes = [P(QwenModel), vp, P(u32), u32, u32, i32]
        L.model_rollback_to.argtypes = [P(QwenModel), u32]
        L.mtp_forward.argtypes = [P(QwenModel), vp, u32, u32, i32]
        L.mtp_forward.restype = i32
        L.mtp_forward_batch.argtypes = [P(QwenModel), vp, P(u32), u32, u32, i32]
        L.mtp_forward_batch.restype = i32
        L.model_sample_greedy.argtypes = [P(f32), u32]
        L.model_sample_greedy.restype = u32
        L.gemv_batch.argtypes = [vp, P(TensorInfo), P(f32), C.c_uint64, i32, P(f32), C.c_uint64]
        L.gemv.argtypes = [vp, P(TensorInfo), P(f32), P(f32)]
        L.gemv_rows.argtypes = [P(TensorInfo), P(f32), P(f32), C.c_uint64, C.c_uint64]
        L.gemv_rows_batch.argtypes = [P(TensorInfo), P(f32), C.c_uint64, i32, P(f32), C.c_uint64,
                                      C.c_uint64, C.c_uint64]
        L.gemv_multi_batch.argtypes = [vp, P(P(TensorInfo)), P(f32), C.c_uint64, i32, P(P(f32)),
                                       P(C.c_uint64), i32]
        L.gemv_multi.argtypes = [vp, P(P(TensorInfo)), P(f32), P(P(f32)), i32]
        for n in ("rmsnorm",):
            getattr(L, n).argtypes = [P(f32), P(f32), P(f32), C.c_uint64, f32]
        L.l2norm.argtypes = [P(f32), P(f32), C.c_uint64, f32]
        for n in ("silu_inplace", "sigmoid_inplace", "softplus_inplace", "softmax_inplace"):
            getattr(L, n).argtypes = [P(f32), C.c_uint64]
        L.qb_last_error.restype = i32
        L.qb_last_error_str.restype = C.c_char_p
        L.qb_prefill.argtypes = [P(QwenModel), P(u32), u32, i32]
        L.qb_prefill.restype = i32
        L.qb_spec_generate.argtypes = [P(QwenModel), u32, u32, P(u32), u32, P(u32), P(u32), u32, P(u32)]
        L.qb_spec_generate.restype = i32
        L.qb_greedy_generate.argtypes = [P(QwenModel), u32, P(u32)]
        L.qb_greedy_generate.restype = i32
        L.qb_last_argmax.argtypes = [P(QwenModel), u32]
        L.qb_last_argmax.restype = u32
        L.qb_last_loop_ms.argtypes = [P(QwenModel)]
        L.qb_last_loop_ms.restype = f32
        L.qb_read_state.argtypes = [P(QwenModel), u32, i32, P(f32), C.c_int64]
        L.qb_read_state.restype = C.c_int64
        L.qb_read_buffer.argtypes = [P(QwenModel), i32, P(f32), C.c_int64]
        L.qb_read_buffer.restype = C.c_int64
        L.qb_reset.argtypes = [P(QwenModel)]
        L.qb_reset.restype = i32
        L.qb_seq_init.argtypes = [P(QwenModel), u32]
        L.qb_seq_init.restype = i32
        L.qb_enable_wide.argtypes = [P(QwenModel)]
        L.qb_enable_wide.restype = i32
        L.qb_seq_prefill.argtypes = [P(QwenModel), u32, P(u32), u32]
        L.qb_seq_prefill.restype = i32
        L.qb_seq_generate.argtypes = [P(QwenModel), u32, u32, P(u32), u32, P(u32), u32, P(u32), P(u32)]
        L.qb_seq_generate.restype = i32
        L.qb_bench.argtypes = [P(QwenModel), i32, u32, u32, P(C.c_double)]
        L.qb_bench.restype = f32
        L.qb_model_init_tp.argtypes = [P(QwenModel), C.c_char_p, u32, i32, i32]
        L.qb_model_init_tp.restype = i32
        L.qb_tp_handle.argtypes = [P(QwenModel), vp, C.c_int64]
        L.qb_tp_handle.restype = C.c_int64
        L.qb_tp_connect.argtypes = [P(QwenModel), vp, C.c_int64]
        L.qb_tp_connect.restype = i32
        L.qb_tp_rows.argtypes = [i32, i32, i32, P(i32), P(i32)]
        L.qb_tp_rows.restype = None
        L.qb_argmax_rows_noalloc.argtypes = [vp, C.c_int64, u32, u32, vp, vp]
        L.qb_argmax_rows_noalloc.restype = i32
        L.sampler_init.argtypes = [f32, f32, u32, f32, C.c_uint64]
        L.sampler_init.restype = P(SamplerT)
        L.sampler_free.argtypes = [P(SamplerT)]
        L.sampler_sample.argtypes = [P(SamplerT), P(f32), u32, P(u32), C.c_size_t]
        L.sampler_sample.restype = u32
        L.qb_sample_generate.argtypes = [P(QwenModel), P(SamplerT), u32, P(u32), C.c_size_t, P(u32)]
        L.qb_sample_generate.restype = i32
        _lib = L
    return _lib


def check():
    L = lib()
    if L.qb_last_error():
        msg = L.qb_last_error_str().decode()
        L.qb_clear_error()
        raise RuntimeError(f"libqwenb200: {msg}")


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _up(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def tensor(data, gtype, ne0, ne1, name=b"t"):
    """gguf_tensor_info_t around a numpy uint8/float32 buffer (kept alive by the caller)."""
    t = TensorInfo()
    t.name = name
    t.n_dims = 2
    t.ne[0], t.ne[1], t.ne[2], t.ne[3] = ne0, ne1, 1, 1
    t.type = gtype
    t.data = data.ctypes.data
    return t


def gemv_batch(t, x, n=None, out=None):
    """out[n][rows] = W x[n][ne0] (include/kernels.h:26) on the GPU."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[0] if n is None else n
    rows = t.ne[1]
    if out is None:
        out = np.zeros((n, rows), np.float32)
    lib().gemv_batch(None, C.byref(t), _fp(x), x.shape[1], n, _fp(out), out.shape[1])
    check()
    return out


def gemv_multi_batch(ts, x, n=None):
    """outs[i][n][rows_i] = W_i x (include/kernels.h:32-34): every matrix reads the
    same x, in one dispatch."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[0] if n is None else n
    outs = [np.zeros((n, t.ne[1]), np.float32) for t in ts]
    W = (C.POINTER(TensorInfo) * len(ts))(*[C.pointer(t) for t in ts])
    O = (C.POINTER(C.c_float) * len(ts))(*[_fp(o) for o in outs])
    ld = (C.c_uint64 * len(ts))(*[o.shape[1] for o in outs])
    lib().gemv_multi_batch(None, W, _fp(x), x.shape[1], n, O, ld, len(ts))
    check()
    return outs


def gemv_multi(ts, x):
    """The single-vector form (include/kernels.h:28-29)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    outs = [np.zeros(t.ne[1], np.float32) for t in ts]
    W = (C.POINTER(TensorInfo) * len(ts))(*[C.pointer(t) for t in ts])
    O = (C.POINTER(C.c_float) * len(ts))(*[_fp(o) for o in outs])
    lib().gemv_multi(None, W, _fp(x), O, len(ts))
    check()
    return outs


def gemv_rows_batch(t, x, r0, r1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros((x.shape[0], t.ne[1]), np.float32)
    lib().gemv_rows_batch(C.byref(t), _fp(x), x.shape[1], x.shape[0], _fp(out), out.shape[1], r0, r1)
    check()
    return out


def sample_greedy(logits):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    r = lib().model_sample_greedy(_fp(logits), logits.size)
    check()
    return r


def argmax_rows_noalloc(logits_ptr, ld, n, rows, out_ptr, stream_ptr=None):
    """qb_argmax_rows_noalloc on device pointers (ints); enqueued on the stream."""
    rc = lib().qb_argmax_rows_noalloc(logits_ptr, ld, n, rows, out_ptr, stream_ptr)
    if rc:
        check()
    return rc


class Sampler:
    """sampler_init / sampler_sample / sampler_free (include/sampler.h) on the GPU."""

    def __init__(self, temp, top_p, top_k, repeat_penalty, seed):
        self.s = lib().sampler_init(temp, top_p, top_k, repeat_penalty, seed)
        if not self.s:
            raise RuntimeError("sampler_init failed")

    @property
    def rng_state(self):
        return self.s.contents.rng_state

    def sample(self, logits, tokens):
        """Returns the token; logits (float32 numpy) are penalised in place."""
        t = np.ascontiguousarray(tokens, np.uint32)
        r = lib().sampler_sample(self.s, _fp(logits), logits.size, _up(t) if t.size else None, t.size)
        check()
        return r

    def close(self):
        if self.s:
            lib().sampler_free(self.s)
            self.s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def op(name, x, w=None, eps=1e-6):
    x = np.ascontiguousarray(x, dtype=np.float32).copy()
    L = lib()
    if name == "rmsnorm":
        out = np.empty_like(x)
        wp = _fp(np.ascontiguousarray(w, np.float32)) if w is not None else None
        L.rmsnorm(_fp(out), _fp(x), wp, x.size, eps)
        x = out
    elif name == "l2norm":
        out = np.empty_like(x)
        L.l2norm(_fp(out), _fp(x), x.size, eps)
        x = out
    else:
        getattr(L, name + "_inplace")(_fp(x), x.size)
    check()
    return x


def tp_rows(rows, rank, world):
    """Row range [r0, r1) of a rows-row matrix held by rank of world (qb_tp_rows)."""
    r0, r1 = C.c_int(0), C.c_int(0)
    lib().qb_tp_rows(rows, rank, world, C.byref(r0), C.byref(r1))
    return r0.value, r1.value


class Model:
    """Owns a qwen_model_t (include/qwen_b200.h) on the current CUDA device.

    With world > 1 the model is this rank's share of a tensor-parallel group
    (qb_model_init_tp): call tp_connect() with every rank's tp_handle() before
    the first forward, then drive all ranks with the same calls."""

    def __init__(self, path, n_ctx, rank=0, world=1):
        self.m = QwenModel()
        if world == 1:
            r = lib().model_init(C.byref(self.m), os.fsencode(path), n_ctx)
        else:
            r = lib().qb_model_init_tp(C.byref(self.m), os.fsencode(path), n_ctx, rank, world)
        if r != 0:
            msg = lib().qb_last_error_str().decode()
            lib().qb_clear_error()
            raise RuntimeError(f"model_init failed: {msg}")
        self.V = self.m.cfg.vocab_size
        self.E = self.m.dims.n_embd
        self.rank, self.world = rank, world

    def tp_handle(self):
        """This rank's IPC handle of its activation arena (bytes)."""
        buf = (C.c_char * 64)()
        n = lib().qb_tp_handle(C.byref(self.m), buf, 64)
        if n <= 0:
            raise RuntimeError("qb_tp_handle failed: " + lib().qb_last_error_str().decode())
        return bytes(buf[:n])

    def tp_connect(self, handles):
        """Map every peer's arena; handles = the tp_handle() of all ranks, rank-ordered."""
        stride = max(len(h) for h in handles)
        blob = b"".join(h.ljust(stride, b"\0") for h in handles)
        buf = C.create_string_buffer(blob, len(blob))
        if lib().qb_tp_connect(C.byref(self.m), buf, stride) != 0:
            raise RuntimeError("qb_tp_connect failed: " + lib().qb_last_error_str().decode())

    def close(self):
        if self.m.eng:
            lib().model_free(C.byref(self.m))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -------- host mirrors --------
    @property
    def pos(self):
        return self.m.pos

    @pos.setter
    def pos(self, v):
        self.m.pos = v

    def logits(self):
        return np.ctypeslib.as_array(self.m.logits, (self.V,)).copy()

    def logits_b(self, B):
        return np.ctypeslib.as_array(self.m.logits_b, (B * self.V,)).reshape(B, self.V).copy()

    def h_save(self, B):
        return np.ctypeslib.as_array(self.m.h_save, (B * self.E,)).reshape(B, self.E).copy()

    def mtp_h(self):
        return np.ctypeslib.as_array(self.m.mtp_h, (self.E,))

    def x(self):
        return np.ctypeslib.as_array(self.m.x, (self.E,)).copy()

    # -------- model.h API --------
    def set_x(self, v):
        np.ctypeslib.as_array(self.m.x, (self.E,))[:] = v

    def layer(self, il, pos):
        """attention_layer / gdn_layer on m->x (the layer kind decides which)."""
        L = C.pointer(self.m.layers[il])
        if self.m.layers[il].is_recurrent:
            lib().gdn_layer(C.byref(self.m), L, None)
        else:
            lib().attention_layer(C.byref(self.m), L, None, pos)
        check()

    def forward(self, tok, pos):
        lib().model_forward(C.byref(self.m), None, tok, pos)
        check()

    def forward_batch(self, toks, pos, ckpt):
        t = np.ascontiguousarray(toks, np.uint32)
        lib().model_forward_batch(C.byref(self.m), None, _up(t), pos, t.size, ckpt)
        check()

    def rollback_to(self, b):
        lib().model_rollback_to(C.byref(self.m), b)
        check()

    def mtp_forward(self, tok, pos, want_logits):
        lib().mtp_forward(C.byref(self.m), None, tok, pos, want_logits)
        check()

    def mtp_forward_batch(self, toks, pos, want_logits):
        t = np.ascontiguousarray(toks, np.uint32)
        lib().mtp_forward_batch(C.byref(self.m), None, _up(t), pos, t.size, want_logits)
        check()

    # -------- device loops --------
    def prefill(self, toks, spec):
        t = np.ascontiguousarray(toks, np.uint32)
        if lib().qb_prefill(C.byref(self.m), _up(t), t.size, spec) != 0:
            check()
            raise RuntimeError("qb_prefill failed")

    def spec_generate(self, n_predict, n_spec=3, forced=None, max_cycles=100000):
        out = np.zeros(n_predict + 8, np.uint32)
        js = np.zeros(max_cycles, np.uint32)
        nc = C.c_uint32()
        f = np.ascontiguousarray(forced if forced is not None else [], np.uint32)
        n = lib().qb_spec_generate(C.byref(self.m), n_predict, n_spec, _up(f) if f.size else None, f.size,
                                   _up(out), _up(js), max_cycles, C.byref(nc))
        if n < 0:
            check()
            raise RuntimeError("qb_spec_generate failed")
        return out[:n].copy(), js[:nc.value].copy()

    def greedy_generate(self, n_predict):
        out = np.zeros(n_predict + 1, np.uint32)
        n = lib().qb_greedy_generate(C.byref(self.m), n_predict, _up(out))
        if n < 0:
            check()
            raise RuntimeError("qb_greedy_generate failed")
        return out[:n].copy()

    def sample_generate(self, sampler, n_predict, history):
        """qb_sample_generate: n_predict tokens drawn on the device (history: the
        tokens the repetition penalty sees)."""
        out = np.zeros(n_predict + 1, np.uint32)
        h = np.ascontiguousarray(history, np.uint32)
        n = lib().qb_sample_generate(C.byref(self.m), sampler.s, n_predict, _up(h) if h.size else None, h.size,
                                     _up(out))
        if n < 0:
            check()
            raise RuntimeError("qb_sample_generate failed")
        return out[:n].copy()

    def enable_wide(self):
        if lib().qb_enable_wide(C.byref(self.m)) != 0:
            check()
            raise RuntimeError("qb_enable_wide failed")

    # ---- multi-sequence decode (qb_seq_*) ----
    def seq_init(self, n_seq):
        if lib().qb_seq_init(C.byref(self.m), n_seq) != 0:
            check()
            raise RuntimeError("qb_seq_init failed")
        self.n_seq = n_seq

    def seq_prefill(self, seq, toks):
        t = np.ascontiguousarray(toks, np.uint32)
        if lib().qb_seq_prefill(C.byref(self.m), seq, _up(t), t.size) != 0:
            check()
            raise RuntimeError("qb_seq_prefill failed")

    def seq_generate(self, n_cycles, n_spec=3, forced=None, cap=None):
        """n_cycles speculative cycles of every sequence: ([tokens of sequence s],
        [accept lengths of sequence s])."""
        S = self.n_seq
        cap = cap or n_cycles * (n_spec + 1) + 8
        out = np.zeros((S, cap), np.uint32)
        cnt = np.zeros(S, np.uint32)
        js = np.zeros((S, n_cycles), np.uint32)
        f = np.ascontiguousarray(forced if forced is not None else [], np.uint32)
        n = lib().qb_seq_generate(C.byref(self.m), n_cycles, n_spec, _up(f) if f.size else None, f.size,
                                  _up(out), cap, _up(cnt), _up(js))
        if n < 0:
            check()
            raise RuntimeError("qb_seq_generate failed")
        return [out[s, :cnt[s]].copy() for s in range(S)], [js[s, :n].copy() for s in range(S)]

    def reset(self):
        if lib().qb_reset(C.byref(self.m)) != 0:
            check()
            raise RuntimeError("qb_reset failed")

    def bench(self, what, arg, iters):
        """(ms per run, algorithmic bytes per run) from qb_bench."""
        b = C.c_double()
        ms = lib().qb_bench(C.byref(self.m), what, arg, iters, C.byref(b))
        if ms < 0:
            check()
            raise RuntimeError("qb_bench failed")
        return float(ms), float(b.value)

    def last_loop_ms(self):
        return lib().qb_last_loop_ms(C.byref(self.m))

    def read_buffer(self, bid, n):
        buf = np.zeros(n, np.float32)
        got = lib().qb_read_buffer(C.byref(self.m), bid, _fp(buf), n)
        if got < 0:
            raise RuntimeError("qb_read_buffer failed")
        return buf[:got]

    def read_state(self, il, which, n):
        buf = np.zeros(n, np.float32)
        got = lib().qb_read_state(C.byref(self.m), il, which, _fp(buf), n)
        if got < 0:
            raise RuntimeError("qb_read_state failed")
        return buf[:got]


# ------------------------------ synthetic weights ------------------------------

class SynthCfg(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_embd", "n_ff", "n_layer", "vocab", "n_head", "n_kv_head",
                                           "head_dim", "rope_dim", "full_attn_interval", "ssm_state",
                                           "ssm_groups", "ssm_v_heads", "d_conv", "n_ctx_train")] + [
        ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("seed", C.c_uint64), ("profile", C.c_uint32),
        ("gain", C.c_float), ("n_threads", C.c_uint32), ("tokenizer", C.c_uint32)]


# Model shapes.  FULL is the benchmark model; the
# smaller ones keep every structural feature for the parity tests.
FULL = dict(n_embd=5120, n_ff=17408, n_layer=64, vocab=248320, n_head=24, n_kv_head=4, head_dim=256,
            rope_dim=64, full_attn_interval=4, ssm_state=128, ssm_groups=16, ssm_v_heads=48, d_conv=4)
TINY = dict(n_embd=512, n_ff=1024, n_layer=4, vocab=2048, n_head=2, n_kv_head=1, head_dim=256,
            rope_dim=64, full_attn_interval=4, ssm_state=128, ssm_groups=2, ssm_v_heads=4, d_conv=4)
SMALL = dict(n_embd=1024, n_ff=2048, n_layer=8, vocab=8192, n_head=4, n_kv_head=2, head_dim=256,
             rope_dim=64, full_attn_interval=4, ssm_state=128, ssm_groups=4, ssm_v_heads=8, d_conv=4)
WIDE4 = dict(FULL, n_layer=4)   # full widths, 3 GDN + 1 attention layer


_synth = None


def synth_lib():
    global _synth
    if _synth is None:
        if not os.path.exists(SYNTH_PATH):
            raise RuntimeError(f"{SYNTH_PATH} missing: run qwen3.8-27b-in-c_b200/build.py")
        L = C.CDLL(SYNTH_PATH)
        L.qb_synth_write.argtypes = [C.c_char_p, C.POINTER(SynthCfg)]
        L.qb_synth_write.restype = C.c_int
        L.qb_synth_file_size.argtypes = [C.POINTER(SynthCfg)]
        L.qb_synth_file_size.restype = C.c_uint64
        L.qb_synth_quant_matrix.argtypes = [C.c_void_p, C.c_int, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float]
        L.qb_synth_quant_matrix.restype = C.c_int
        L.qb_synth_normal_f32.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64]
        _synth = L
    return _synth


def synth_cfg(shape, seed=0, profile=0, gain=1.0, rope_theta=1e7, rms_eps=1e-6, n_threads=0, tokenizer=0):
    c = SynthCfg(**shape)
    c.tokenizer = tokenizer
    c.n_ctx_train = 262144
    c.rope_theta = rope_theta
    c.rms_eps = rms_eps
    c.seed = seed
    c.profile = profile
    c.gain = gain
    c.n_threads = n_threads
    return c


def write_synth_gguf(path, shape, seed=0, profile=0, **kw):
    c = synth_cfg(shape, seed=seed, profile=profile, **kw)
    r = synth_lib().qb_synth_write(os.fsencode(path), C.byref(c))
    if r != 0:
        raise RuntimeError(f"qb_synth_write failed ({r})")
    return path


def synth_matrix(gtype, rows, K, seed=0, d_sigma=0.02):
    buf = np.zeros(rows * row_bytes(gtype, K), np.uint8)
    r = synth_lib().qb_synth_quant_matrix(buf.ctypes.data, gtype, rows, K, seed, d_sigma)
    if r != 0:
        raise RuntimeError("qb_synth_quant_matrix failed")
    return buf


def synth_normal(n, seed):
    out = np.zeros(n, np.float32)
    synth_lib().qb_synth_normal_f32(out.ctypes.data, n, seed)
    return out
