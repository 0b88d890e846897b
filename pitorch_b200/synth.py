"""Seeded synthetic checkpoints, prompts and token sequences.

The reference's real checkpoints (stories15M/42M/110M) are not available, so
every benchmark and parity test runs on llama2.c-format blobs whose tensors
are i.i.d. N(0, 0.02) float32 drawn in file order from
``numpy.random.default_rng(seed)``. The header follows the reference loader
(pitorch/model/llama2.c:9-19): ``dim, hidden_dim, n_layers, n_heads,
n_kv_heads, vocab_size, seq_len``; a positive vocab means the classifier is
tied to the embedding (llama2.c:166). The freq_cis region, which the loader
skips (llama2.c:164-165), is zero-filled.
"""
import numpy as np

# name -> (dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab, seq_len)
CONFIGS = {
    "tiny": (64, 176, 2, 4, 4, 1024, 64),
    "stories15M": (288, 768, 6, 6, 6, 32000, 256),
    "stories42M": (512, 1376, 8, 8, 8, 32000, 1024),
    "stories110M": (768, 2048, 12, 12, 12, 32000, 1024),
}

DEFAULT_SEED = 1234


def param_count(cfg):
    dim, hidden, L, nh, nkv, V, seq = cfg
    kvd = nkv * (dim // nh)
    return (V * dim + L * dim + L * dim * dim + 2 * L * kvd * dim + L * dim * dim
            + L * dim + 3 * L * hidden * dim + dim)


def blob_bytes(cfg):
    dim, hidden, L, nh, nkv, V, seq = cfg
    return 28 + 4 * (param_count(cfg) + seq * (dim // nh))


def make_blob(cfg, seed=DEFAULT_SEED, std=0.02):
    """Return a llama2.c .bin image (bytes) for ``cfg`` with a tied classifier."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    dim, hidden, L, nh, nkv, V, seq = cfg
    n = param_count(cfg)
    hd = dim // nh
    rng = np.random.default_rng(seed)
    out = np.empty(7 + n + seq * hd, dtype=np.float32)
    out[:7].view(np.int32)[:] = np.array([dim, hidden, L, nh, nkv, V, seq], dtype=np.int32)
    w = out[7:7 + n]
    rng.standard_normal(out=w, dtype=np.float32)
    w *= np.float32(std)
    out[7 + n:] = 0.0
    return out.tobytes()


def make_prompt(vocab, n=8, seed=DEFAULT_SEED):
    """n prompt tokens uniform over [3, vocab-1] (3..31999 at vocab 32000)."""
    return np.random.default_rng(seed + 1).integers(3, vocab, size=n).astype(np.int32)


def make_tokens(vocab, T, seed=DEFAULT_SEED):
    """T training tokens uniform over [0, vocab)."""
    return np.random.default_rng(seed + 2).integers(0, vocab, size=T).astype(np.int32)
