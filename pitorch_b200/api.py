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


class pt_dist_t(C.Structure):
    _fields_ = [("rank", C.c_int), ("world_size", C.c_int), ("l_start", C.c_int), ("l_end", C.c_int),
                ("has_embed", C.c_int), ("has_head", C.c_int), ("comm", C.c_void_p),
                ("timeout_ms", C.c_int)]


class pt_token_index_t(C.Structure):
    _fields_ = [("str", C.c_char_p), ("id", C.c_int)]


class pt_tokenizer_t(C.Structure):
    _fields_ = [("vocab", C.c_void_p), ("vocab_scores", f32p), ("vocab_size", C.c_int),
                ("max_token_length", C.c_int), ("sorted_ready", C.c_int),
                ("sorted_vocab", C.POINTER(pt_token_index_t))]


class pt_sampler_t(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("temperature", C.c_float), ("topp", C.c_float),
                ("rng_state", C.c_uint64)]


def declare_text(L):
    """Signatures of the text layer (include/pt_text.h). Separate from
    declare() because the reference's own build exports the same names."""
    P = C.POINTER
    _sig(L, "pt_tokenizer_init", None, P(pt_tokenizer_t), C.c_void_p, C.c_int)
    _sig(L, "pt_load_tokenizer", None, P(pt_tokenizer_t), C.c_void_p, C.c_int)
    _sig(L, "pt_tokenizer_free", None, P(pt_tokenizer_t))
    _sig(L, "pt_decode", C.c_char_p, P(pt_tokenizer_t), C.c_int, C.c_int)
    _sig(L, "pt_encode", None, P(pt_tokenizer_t), C.c_char_p, C.c_int, C.c_int, i32p, i32p)
    _sig(L, "pt_sampler_init", None, P(pt_sampler_t), C.c_int, C.c_float, C.c_float, C.c_uint64)
    _sig(L, "pt_sample", C.c_int, P(pt_sampler_t), f32p)
    _sig(L, "pt_generate", None, P(pt_config_t), P(pt_weights_t), P(pt_state_t), P(pt_tokenizer_t),
         P(pt_sampler_t), C.c_char_p, C.c_int, vp)
    return L


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
    _sig(L, "pt_save_weights", C.c_int, ctx, C.c_char_p)
    _sig(L, "pt_ptc_ctx", vp, ctx)
    _sig(L, "pt_ptc_decoder", vp, ctx)
    _sig(L, "pt_ptc_trainer", vp, ctx)
    for name in ("ptc_trainer_zero_grads", "ptc_trainer_fwd_embed", "ptc_trainer_bwd_head",
                 "ptc_trainer_bwd_embed", "ptc_trainer_sync"):
        _sig(L, name, None, vp)
    _sig(L, "ptc_trainer_fwd_head", C.c_float, vp)
    _sig(L, "ptc_trainer_set_tokens", None, vp, i32p, C.c_int)
    _sig(L, "ptc_trainer_fwd_layers", None, vp, C.c_int, C.c_int)
    _sig(L, "ptc_trainer_bwd_layers", None, vp, C.c_int, C.c_int)
    _sig(L, "ptc_trainer_sgd_layers", None, vp, C.c_float, C.c_int, C.c_int)
    _sig(L, "ptc_trainer_sgd_head", None, vp, C.c_float)
    _sig(L, "ptc_trainer_set_microbatches", None, vp, C.c_int)
    _sig(L, "ptc_trainer_select", None, vp, C.c_int)
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
    dist = P(pt_dist_t)
    _sig(L, "pt_dist_setup", None, dist, P(pt_shard_info_t), C.c_int, C.c_int)
    _sig(L, "pt_dist_setup_ctx", C.c_int, dist, ctx, P(pt_shard_info_t), C.c_int, C.c_int)
    _sig(L, "pt_dist_transport", C.c_int, dist)
    _sig(L, "pt_dist_comm_size", C.c_int, dist)
    _sig(L, "pt_dist_vocab_parallel", C.c_int, ctx, dist)
    _sig(L, "pt_dist_is_vocab_parallel", C.c_int, dist)
    _sig(L, "pt_dist_train_step_mb", pt_dist_result_t, ctx, dist, i32p, C.c_int, C.c_int, C.c_float)
    _sig(L, "pt_dist_forward_step", C.c_int, ctx, dist, C.c_int)
    _sig(L, "pt_dist_generate_greedy", C.c_int, ctx, dist, i32p, C.c_int, C.c_int, i32p)
    _sig(L, "pt_dist_train_step", pt_dist_result_t, ctx, dist, i32p, C.c_int, C.c_float)
    _sig(L, "pt_dist_allreduce_grads_avg", C.c_int, ctx, dist)
    _sig(L, "pt_dist_max_float", C.c_float, ctx, dist, C.c_float)
    _sig(L, "pt_dist_free", None, dist)
    _sig(L, "pt_dist_set_verbose", None, dist, C.c_int)
    _sig(L, "pt_dist_ring_sync", C.c_int, dist)
    _sig(L, "pt_dist_rendezvous", C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int, C.c_int,
         C.POINTER(C.c_ubyte))
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
    _sig(L, "ptc_decoder_trace", C.c_size_t, vp, C.c_int)
    _sig(L, "ptc_decoder_read_trace", C.c_size_t, vp, C.POINTER(C.c_ulonglong), C.c_size_t)
    _sig(L, "ptc_gemm_counters", None, C.POINTER(C.c_longlong))
    _sig(L, "ptc_decoder_enqueue_embed", None, vp, C.c_int)
    _sig(L, "ptc_decoder_enqueue_layers", None, vp, C.c_int, C.c_int, C.c_int)
    _sig(L, "ptc_decoder_enqueue_head", None, vp)
    _sig(L, "ptc_decoder_enqueue_kernel", None, vp, C.c_int, C.c_int, C.c_int)
    _sig(L, "ptc_decoder_launches_per_step", C.c_int, vp)
    _sig(L, "ptc_decoder_fetch_next", C.c_int, vp, f32p)
    _sig(L, "ptc_decoder_step", C.c_int, vp, C.c_int, C.c_int, f32p)
    _sig(L, "ptc_read_probe", None, vp, C.c_size_t, vp, vp)
    _sig(L, "ptc_mailbox_alloc", vp, vp, C.c_int)
    _sig(L, "ptc_mailbox_free", None, vp)
    _sig(L, "ptc_hop_send", None, vp, vp, vp, vp, vp, C.c_int)
    _sig(L, "ptc_hop_recv", None, vp, vp, vp, vp, vp, C.c_int, vp, C.c_longlong)
    _sig(L, "ptc_timer_create", vp, vp)
    _sig(L, "ptc_timer_start", None, vp)
    _sig(L, "ptc_timer_stop", None, vp)
    _sig(L, "ptc_timer_ms", C.c_float, vp)
    _sig(L, "ptc_timer_destroy", None, vp)
    _sig(L, "ptc_capture_begin", None, vp)
    _sig(L, "ptc_capture_end", vp, vp)
    _sig(L, "ptc_graph_launch", None, vp)
    _sig(L, "ptc_graph_destroy", None, vp)
    _sig(L, "ptc_d2d", None, vp, vp, vp, C.c_size_t)
    return declare_text(L)


def fp(a):
    return a.ctypes.data_as(f32p)


def ip(a):
    return a.ctypes.data_as(i32p)


class Context:
    """A ``pt_context_t`` initialised from a .bin image (``pt_pi_init``), or
    from a SHRD shard (``pt_pi_init_shard``) when ``shard=True``."""

    def __init__(self, blob, max_T=0, device=-1, arena_bytes=0, shard=False):
        from . import lib
        self.L = lib()
        # The context's weight pointers point into this buffer; keep it alive.
        self._blob = C.create_string_buffer(bytes(blob), len(blob))
        self.ctx = pt_context_t()
        self.shard = pt_shard_info_t()
        if shard:
            self.L.pt_pi_init_shard(C.byref(self.ctx), C.byref(self.shard), C.cast(self._blob, C.c_void_p),
                                    device, max_T, arena_bytes)
        else:
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


def make_shard(full_blob, rank, world):
    """Cut rank's SHRD shard out of a full .bin image (pt_make_shard)."""
    from . import lib
    L = lib()
    src = C.create_string_buffer(bytes(full_blob), len(full_blob))
    cap = len(full_blob) + 64
    out = C.create_string_buffer(cap)
    n = L.pt_make_shard(C.cast(src, C.c_void_p), rank, world, C.cast(out, C.c_void_p), cap)
    if n == 0:
        raise ValueError("pt_make_shard failed")
    return out.raw[:n]


class Pipeline:
    """One rank of the layer pipeline: a shard context plus its ring link."""

    def __init__(self, full_blob, rank, world, device, max_T=0):
        from . import lib
        self.L = lib()
        self.rank, self.world = rank, world
        self.ctx = Context(make_shard(full_blob, rank, world), max_T=max_T, device=device, shard=True)
        self.dist = pt_dist_t()
        rc = self.L.pt_dist_setup_ctx(C.byref(self.dist), C.byref(self.ctx.ctx), C.byref(self.ctx.shard),
                                      rank, world)
        if rc != 0:
            raise RuntimeError(f"rank {rank}: pipeline rendezvous failed")

    @property
    def is_head(self):
        return bool(self.dist.has_embed and self.dist.has_head)

    def vocab_parallel(self):
        """Split the classifier over all ranks (pt_dist_vocab_parallel; every
        rank calls it)."""
        if self.L.pt_dist_vocab_parallel(C.byref(self.ctx.ctx), C.byref(self.dist)) != 0:
            raise RuntimeError(f"rank {self.rank}: vocab-parallel classifier set-up failed")

    def generate_greedy(self, prompt, n_pos):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_pos, dtype=np.int32)
        rc = self.L.pt_dist_generate_greedy(C.byref(self.ctx.ctx), C.byref(self.dist), ip(prompt), len(prompt),
                                            n_pos, ip(out))
        if rc != 0:
            raise RuntimeError("pipeline generate failed")
        return out

    def forward_step(self, token):
        return self.L.pt_dist_forward_step(C.byref(self.ctx.ctx), C.byref(self.dist), int(token))

    def decode_greedy(self, prompt, n_pos, logit_rows=()):
        """Host-driven pipeline decode through pt_dist_forward_step. On the
        head rank, logit_rows selects positions whose host logits are kept
        (returned as a dict after the tokens when given)."""
        self.ctx.reset_kv()
        toks = np.zeros(n_pos, dtype=np.int32)
        kept = {}
        tok = int(prompt[0])
        for p in range(n_pos):
            nxt = self.forward_step(tok)
            if nxt < 0:
                raise RuntimeError("pipeline step failed")
            if self.is_head:
                if p in logit_rows:
                    kept[p] = self.ctx.logits()
                nxt = int(prompt[p + 1]) if p + 1 < len(prompt) else nxt
                toks[p] = nxt
                tok = nxt
        return (toks, kept) if logit_rows else toks

    def train_step(self, tokens, lr):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        r = self.L.pt_dist_train_step(C.byref(self.ctx.ctx), C.byref(self.dist), ip(tokens), len(tokens),
                                      C.c_float(lr))
        if r.total_ms == 0:
            raise RuntimeError("pipeline train step failed")
        return r.loss

    def train_step_mb(self, tokens, n_mb, lr):
        """GPipe step over n_mb microbatches (tokens: n_mb * T ids)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        T = len(tokens) // n_mb
        r = self.L.pt_dist_train_step_mb(C.byref(self.ctx.ctx), C.byref(self.dist), ip(tokens), T, n_mb,
                                         C.c_float(lr))
        if r.total_ms == 0:
            raise RuntimeError("pipeline microbatch step failed")
        return r.loss

    def max_over_ranks(self, v):
        return float(self.L.pt_dist_max_float(C.byref(self.ctx.ctx), C.byref(self.dist), C.c_float(v)))

    def close(self):
        self.L.pt_dist_free(C.byref(self.dist))
        self.ctx.close()
