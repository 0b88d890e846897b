"""ctypes mirror of the pitorch C API declared in include/*.h.

Struct layouts follow the headers field for field (checked against the C
compiler by tests/test_abi.py). ``Context`` wraps a ``pt_context_t`` the way
the reference's C callers use one (pt_host_init / pt_forward_step /
pt_train_step / pt_free).
"""
import ctypes as C

import numpy as np

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int)
vp = C.c_void_p


class pt_config_t(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "seq_len")]


_W = ("token_embedding", "rms_att_weight", "wq", "wk", "wv", "wo", "rms_ffn_weight",
      "w1", "w2", "w3", "rms_final_weight", "wcls")


class pt_weights_t(C.Structure):
    _fields_ = [(n, f32p) for n in _W]


class pt_state_t(C.Structure):
    _fields_ = [(n, f32p) for n in
                ("x", "xb", "xb2", "q", "k", "v", "hb", "hb2", "att", "logits",
                 "key_cache", "value_cache")]


class pt_activations_t(C.Structure):
    _fields_ = [(n, f32p) for n in
                ("residuals", "residuals_att", "xb_att", "q", "k", "v", "att", "att_out",
                 "xb_ffn", "hb", "hb2", "x_final", "logits", "scratch")] + [("T", C.c_int)]


class pt_grads_t(C.Structure):
    _fields_ = [(n, f32p) for n in _W] + [("_mem", f32p), ("_n_params", C.c_int)]


class pt_backward_buf_t(C.Structure):
    _fields_ = [(n, f32p) for n in
                ("d_res", "d_aout", "d_q", "d_k", "d_v", "d_logit", "d_xb", "d_qpre", "d_kpre",
                 "d_hid", "d_hid2", "sh", "d_att_s", "d_pre_sm", "w_transpose", "d_temp",
                 "d_logit_all", "drt_wo_all", "d_qpre_all", "d_kpre_all", "sh_all", "d_hid_all",
                 "d_hid2_all", "drt_ffn_all")]


MATVEC_FN = C.CFUNCTYPE(None, f32p, f32p, f32p, C.c_int, C.c_int)


class pt_context_t(C.Structure):
    _fields_ = [("cfg", pt_config_t), ("w", pt_weights_t), ("shared_weights", C.c_int),
                ("matvec", vp), ("state", pt_state_t), ("pos", C.c_int),
                ("acts", pt_activations_t), ("grads", pt_grads_t), ("bb", pt_backward_buf_t),
                ("max_T", C.c_int), ("trace", vp), ("num_qpus", C.c_int),
                ("dev", vp), ("sync_logits", C.c_int)]


class pt_shard_info_t(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("rank", "world_size", "l_start", "l_end", "n_local", "has_embed", "has_head",
                 "n_layers_global")]


class pt_dist_result_t(C.Structure):
    _fields_ = [("loss", C.c_float), ("total_ms", C.c_uint)]


def _sig(L, name, res, *args):
    f = getattr(L, name, None)
    if f is None:
        return
    f.restype = res
    f.argtypes = list(args)


def declare(L):
    P = C.POINTER
    ctx = P(pt_context_t)
    _sig(L, "pt_host_init", None, ctx, C.c_void_p, C.c_int)
    _sig(L, "pt_pi_init", None, ctx, C.c_void_p, C.c_int, C.c_int, C.c_uint)
    _sig(L, "pt_pi_init_shard", None, ctx, P(pt_shard_info_t), C.c_void_p, C.c_int, C.c_int, C.c_uint)
    _sig(L, "pt_free", None, ctx)
    _sig(L, "pt_forward_step", C.c_int, ctx, C.c_int)
    _sig(L, "pt_reset_kv", None, ctx)
    _sig(L, "pt_print_config", None, ctx)
    _sig(L, "pt_train_step", C.c_float, ctx, i32p, C.c_int, C.c_float)
    _sig(L, "pt_generate_greedy", None, ctx, i32p, C.c_int, C.c_int, i32p)
    _sig(L, "pt_sync_weights", None, ctx)
    _sig(L, "pt_sync_grads", None, ctx)
    _sig(L, "pt_ptc_ctx", vp, ctx)
    _sig(L, "pt_ptc_decoder", vp, ctx)
    _sig(L, "pt_load_config", None, P(pt_config_t), C.c_void_p)
    _sig(L, "pt_load_weights", None, P(pt_weights_t), P(pt_config_t), C.c_void_p)
    _sig(L, "pt_file_size", C.c_uint, C.c_void_p)
    _sig(L, "pt_alloc_state", None, P(pt_state_t), P(pt_config_t))
    _sig(L, "pt_free_state", None, P(pt_state_t))
    _sig(L, "pt_forward", None, P(pt_config_t), P(pt_weights_t), P(pt_state_t), C.c_int, C.c_int, vp)
    _sig(L, "pt_forward_embed", None, P(pt_weights_t), f32p, C.c_int, C.c_int)
    _sig(L, "pt_forward_layers_range", None, P(pt_config_t), P(pt_weights_t), P(pt_state_t),
         C.c_int, C.c_int, C.c_int, vp)
    _sig(L, "pt_forward_head", None, P(pt_config_t), P(pt_weights_t), P(pt_state_t), vp)
    _sig(L, "pt_argmax", C.c_int, f32p, C.c_int)
    _sig(L, "pt_matvec_gpu", None, f32p, f32p, f32p, C.c_int, C.c_int)
    _sig(L, "pt_load_shard_header", None, P(pt_config_t), P(pt_shard_info_t), C.c_void_p)
    _sig(L, "pt_shard_file_size", C.c_uint, C.c_void_p)
    _sig(L, "pt_make_shard", C.c_ulong, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_ulong)
    acts, grads, bb, cfgp, wp = P(pt_activations_t), P(pt_grads_t), P(pt_backward_buf_t), P(pt_config_t), P(pt_weights_t)
    _sig(L, "pt_zero_grads", None, grads)
    _sig(L, "pt_forward_train", C.c_float, cfgp, wp, acts, i32p, C.c_int, vp, vp)
    _sig(L, "pt_backward", None, cfgp, wp, grads, acts, bb, i32p, C.c_int, vp, vp)
    _sig(L, "pt_sgd_update", None, wp, grads, C.c_float, cfgp)
    _sig(L, "pt_sgd_update_layers", None, wp, grads, C.c_float, cfgp, C.c_int, C.c_int)
    _sig(L, "pt_sgd_update_head", None, wp, grads, C.c_float, cfgp)
    _sig(L, "pt_forward_train_embed", None, wp, acts, i32p, C.c_int, C.c_int)
    _sig(L, "pt_forward_train_layers_range", None, cfgp, wp, acts, C.c_int, C.c_int, C.c_int, vp, vp)
    _sig(L, "pt_forward_train_head", C.c_float, cfgp, wp, acts, i32p, C.c_int, vp, vp)
    _sig(L, "pt_backward_head", None, cfgp, wp, grads, acts, bb, i32p, C.c_int, vp, vp)
    _sig(L, "pt_backward_layers_range", None, cfgp, wp, grads, acts, bb, C.c_int, C.c_int, C.c_int, vp, vp)
    _sig(L, "pt_backward_embed", None, grads, bb, i32p, C.c_int, C.c_int)
    # thin C ABI (ptc.h)
    _sig(L, "ptc_device_count", C.c_int)
    _sig(L, "ptc_create", vp, C.c_int, C.c_size_t)
    _sig(L, "ptc_destroy", None, vp)
    _sig(L, "ptc_alloc", vp, vp, C.c_size_t)
    _sig(L, "ptc_stream", vp, vp)
    _sig(L, "ptc_sync", None, vp)
    _sig(L, "ptc_h2d", None, vp, vp, vp, C.c_size_t)
    _sig(L, "ptc_d2h", None, vp, vp, vp, C.c_size_t)
    _sig(L, "ptc_memset", None, vp, vp, C.c_int, C.c_size_t)
    _sig(L, "ptc_sm_count", C.c_int, vp)
    _sig(L, "ptc_matvec", None, vp, vp, vp, C.c_int, C.c_int, vp)
    _sig(L, "ptc_matvec_host", None, f32p, f32p, f32p, C.c_int, C.c_int)
    _sig(L, "ptc_sgemm_noalloc", C.c_int, C.c_int, C.c_int, C.c_int, vp, C.c_int, C.c_int, vp, C.c_int,
         C.c_int, vp, C.c_int, C.c_int, vp)
    _sig(L, "ptc_sgemm", None, C.c_int, C.c_int, C.c_int, vp, C.c_int, C.c_int, vp, C.c_int, C.c_int,
         vp, C.c_int, C.c_int, vp, C.c_size_t, vp)
    _sig(L, "ptc_decoder_generate_begin", None, vp, i32p, C.c_int)
    _sig(L, "ptc_decoder_enqueue_steps", None, vp, C.c_int)
    _sig(L, "ptc_decoder_read_tokens", None, vp, i32p, C.c_int)
    _sig(L, "ptc_decoder_reset", None, vp)
    _sig(L, "ptc_decoder_is_persistent", C.c_int, vp)
    _sig(L, "ptc_decoder_trace", None, vp, C.c_int)
    _sig(L, "ptc_decoder_read_trace", C.c_int, vp, C.POINTER(C.c_ulonglong), C.c_int)
    _sig(L, "ptc_decoder_enqueue_embed", None, vp, C.c_int)
    _sig(L, "ptc_decoder_enqueue_layers", None, vp, C.c_int, C.c_int, C.c_int)
    _sig(L, "ptc_decoder_enqueue_head", None, vp)
    _sig(L, "ptc_decoder_fetch_next", C.c_int, vp, f32p)
    _sig(L, "ptc_decoder_step", C.c_int, vp, C.c_int, C.c_int, f32p)
    _sig(L, "ptc_timer_create", vp, vp)
    _sig(L, "ptc_timer_start", None, vp)
    _sig(L, "ptc_timer_stop", None, vp)
    _sig(L, "ptc_timer_ms", C.c_float, vp)
    _sig(L, "ptc_timer_destroy", None, vp)


def fp(a):
    return a.ctypes.data_as(f32p)


def ip(a):
    return a.ctypes.data_as(i32p)


class Context:
    """A ``pt_context_t`` initialised from a .bin image (``pt_pi_init``)."""

    def __init__(self, blob, max_T=0, device=-1, arena_bytes=0):
        from . import lib
        self.L = lib()
        # The context's weight pointers point into this buffer; keep it alive.
        self._blob = C.create_string_buffer(bytes(blob), len(blob))
        self.ctx = pt_context_t()
        self.L.pt_pi_init(C.byref(self.ctx), C.cast(self._blob, C.c_void_p), device, max_T, arena_bytes)
        self.cfg = self.ctx.cfg
        self._open = True

    @property
    def pos(self):
        return self.ctx.pos

    def forward_step(self, token):
        return self.L.pt_forward_step(C.byref(self.ctx), int(token))

    def logits(self):
        return np.ctypeslib.as_array(self.ctx.state.logits, shape=(self.cfg.vocab_size,)).copy()

    def x(self):
        return np.ctypeslib.as_array(self.ctx.state.x, shape=(self.cfg.dim,)).copy()

    def reset_kv(self):
        self.L.pt_reset_kv(C.byref(self.ctx))

    def generate_greedy(self, prompt, n_pos):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_pos, dtype=np.int32)
        self.L.pt_generate_greedy(C.byref(self.ctx), ip(prompt), len(prompt), n_pos, ip(out))
        return out

    def decode_greedy(self, prompt, n_pos, want_logits=False):
        """Host-driven decode through pt_forward_step (the drop-in path)."""
        self.reset_kv()
        toks = np.zeros(n_pos, dtype=np.int32)
        logits = np.zeros((n_pos, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        tok = int(prompt[0])
        for p in range(n_pos):
            nxt = self.forward_step(tok)
            if want_logits:
                logits[p] = self.logits()
            nxt = int(prompt[p + 1]) if p + 1 < len(prompt) else nxt
            toks[p] = nxt
            tok = nxt
        return (toks, logits) if want_logits else toks

    def train_step(self, tokens, lr):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        return float(self.L.pt_train_step(C.byref(self.ctx), ip(tokens), len(tokens), C.c_float(lr)))

    def ptc_ctx(self):
        return self.L.pt_ptc_ctx(C.byref(self.ctx))

    def ptc_decoder(self):
        return self.L.pt_ptc_decoder(C.byref(self.ctx))

    def blob(self):
        self.L.pt_sync_weights(C.byref(self.ctx))
        return bytes(self._blob.raw)

    def close(self):
        if self._open:
            self.L.pt_free(C.byref(self.ctx))
            self._open = False

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
