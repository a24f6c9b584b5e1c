"""Layer builders with the reference's signatures, validation and weight
draws, producing the same layer dicts (the data contract the attention path
executes; nn/layers.py:332-349, nn/io.py:9-19).

Each builder appends to `self.layers` and keeps the reference's width
bookkeeping (`_last_width`, `_residual_stack`), so they bind onto any
container with those attributes -- AttentionNet here, or the reference's own
NeuralNet. Weights come from NumPy's legacy global RNG in the reference's
order (init_weights, nn/weight_init.py:11-46), so `set_seed(s)` followed by the
same builder calls gives bit-identical weights.
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional

import numpy as np

from .backend import default_dtype

NORMAL_INIT_STD = 0.1          # core/constants.py:67
SINUSOIDAL_BASE = 10000.0      # core/constants.py:70


# ------------------------------------------------------------------- init
def init_weights(n_in: int, n_out: int, method: str = "xavier_uniform",
                 std: Optional[float] = None):
    """(weights (n_out, n_in), zero bias (n_out,)), nn/weight_init.py:11-46."""
    dt = default_dtype()
    if method == "xavier_uniform":
        limit = np.sqrt(6 / (n_in + n_out))
        w = np.random.uniform(-limit, limit, (n_out, n_in)).astype(dt)
    elif method == "xavier_normal":
        w = np.random.normal(0, np.sqrt(2 / (n_in + n_out)), (n_out, n_in)).astype(dt)
    elif method == "he_uniform":
        limit = np.sqrt(6 / n_in)
        w = np.random.uniform(-limit, limit, (n_out, n_in)).astype(dt)
    elif method == "he_normal":
        w = np.random.normal(0, np.sqrt(2 / n_in), (n_out, n_in)).astype(dt)
    elif method == "normal":
        w = np.random.normal(0, NORMAL_INIT_STD if std is None else std, (n_out, n_in)).astype(dt)
    elif method == "orthogonal":
        w = np.random.normal(0, 1, (n_out, n_in)).astype(dt)
        u, _, vt = np.linalg.svd(w, full_matrices=False)
        w = u @ vt
    elif method == "zeros":
        w = np.zeros((n_out, n_in), dtype=dt)
    elif method == "ones":
        w = np.ones((n_out, n_in), dtype=dt)
    else:
        raise ValueError(f"Unknown initialization method: {method}")
    return w, np.zeros(n_out, dtype=dt)


def init_embedding_weights(vocab_size: int, embed_dim: int, method: str = "normal",
                           std: Optional[float] = None):
    """Embedding table (vocab_size, embed_dim), nn/weight_init.py:114-133."""
    dt = default_dtype()
    if method == "normal":
        s = NORMAL_INIT_STD if std is None else std
        return np.random.normal(0, s, (vocab_size, embed_dim)).astype(dt)
    if method == "xavier_uniform":
        limit = np.sqrt(6 / (vocab_size + embed_dim))
        return np.random.uniform(-limit, limit, (vocab_size, embed_dim)).astype(dt)
    if method == "xavier_normal":
        s = np.sqrt(2 / (vocab_size + embed_dim))
        return np.random.normal(0, s, (vocab_size, embed_dim)).astype(dt)
    if method == "zeros":
        return np.zeros((vocab_size, embed_dim), dtype=dt)
    raise ValueError(f"Unknown embedding init method: {method}")


# -------------------------------------------------------------- helpers
def _require_width(self: Any, what: str) -> int:
    if self._last_width is None:
        raise ValueError(
            f"Cannot auto-infer input size for {what}: no previous layer to infer it from. "
            f"Pass the size explicitly for the first layer in the model.")
    return self._last_width


def _validate_num_kv_heads(num_heads: int, num_kv_heads: Optional[int], where: str) -> int:
    """nn/layers.py:210-220."""
    if num_kv_heads is None:
        return num_heads
    if num_kv_heads < 1 or num_heads % num_kv_heads != 0:
        raise ValueError(
            f"{where}: num_kv_heads={num_kv_heads} must be >= 1 and divide "
            f"num_heads={num_heads} evenly (each K/V head is shared by exactly "
            f"num_heads // num_kv_heads query heads).")
    return num_kv_heads


def _set_width(self: Any, width: int) -> None:
    self._last_width = width
    if hasattr(self, "_last_spatial"):
        self._last_spatial = None
    if hasattr(self, "_last_spatial_1d"):
        self._last_spatial_1d = None


# ----------------------------------------------------------- attention
ATTENTION_KERNELS = ("softmax", "linear", "performer")  # nn/attention_kernels.py:20


def make_projection(num_features: int, head_dim: int) -> np.ndarray:
    """Performer random features (nn/attention_kernels.py:23-35): orthogonal
    rows in blocks of head_dim (the transpose of a QR factor of a Gaussian
    square), scaled to the norms of Gaussian rows. Draws from the global RNG
    in the reference's order: one head_dim x head_dim Gaussian per block, then
    one (num_features, head_dim) Gaussian for the norms."""
    n_blocks = -(-num_features // head_dim)
    rows = np.concatenate([np.linalg.qr(np.random.randn(head_dim, head_dim))[0].T
                           for _ in range(n_blocks)], axis=0)[:num_features]
    scale = np.linalg.norm(np.random.randn(num_features, head_dim), axis=1)
    return (rows * scale[:, None]).astype(default_dtype())


def _validate_attention_kernel(kernel: str, positional_scheme: str, window_size,
                               dropout: float, head_dim: int, num_features) -> Optional[np.ndarray]:
    """nn/layers.py:223-253: a linearized kernel builds no score matrix, so
    ALiBi, a window and attention dropout are rejected; every linearized
    kernel draws a projection (only the Performer uses it) before the layer's
    weights, which keeps the RNG stream in the reference's order."""
    if kernel not in ATTENTION_KERNELS:
        raise ValueError(f"Unknown attention_kernel {kernel!r}. Expected one of {ATTENTION_KERNELS}.")
    if kernel == "softmax":
        return None
    for name, bad, why in (
            ("positional_scheme='alibi'", positional_scheme == "alibi",
             "ALiBi is an additive bias on the score matrix"),
            ("window_size", window_size is not None, "a sliding window is a mask on the score matrix"),
            ("dropout", dropout > 0, "attention dropout is a mask on the softmax weights")):
        if bad:
            raise ValueError(
                f"attention_kernel={kernel!r} is incompatible with {name}: {why}, and linearized "
                "attention never materializes one. Use attention_kernel='softmax' if you need it.")
    return make_projection(num_features or head_dim * 4, head_dim)


def add_multihead_attention(self: Any, embed_dim: Optional[int] = None, num_heads: int = 4,
                            dropout: float = 0.0, init_method: str = "xavier_uniform",
                            causal: bool = False, positional_scheme: str = "absolute",
                            num_kv_heads: Optional[int] = None,
                            window_size: Optional[int] = None,
                            attention_kernel: str = "softmax",
                            num_features: Optional[int] = None,
                            sparse_pattern: Optional[Dict[str, int]] = None,
                            tiled_block_size: Optional[int] = None) -> None:
    """Multi-head self-attention, nn/layers.py:256-354. attention_kernel
    "softmax" runs the fused softmax kernels; "linear" (elu + 1) and
    "performer" (FAVOR+) run the linearized-attention kernels; a
    sparse_pattern (nn/sparse_attention.py) runs the softmax kernel over the
    pattern's key tiles only. tiled_block_size is accepted (the softmax kernel
    always streams) and validated as the reference does."""
    if embed_dim is None:
        embed_dim = _require_width(self, "add_multihead_attention")
    if embed_dim % num_heads != 0:
        raise ValueError("embed_dim must be divisible by num_heads")
    head_dim = embed_dim // num_heads
    num_kv_heads = _validate_num_kv_heads(num_heads, num_kv_heads, "add_multihead_attention")
    kv_dim = num_kv_heads * head_dim
    if window_size is not None and window_size < 0:
        raise ValueError(f"window_size must be >= 0 or None, got {window_size}")
    omega = _validate_attention_kernel(attention_kernel, positional_scheme, window_size,
                                       dropout, head_dim, num_features)
    if sparse_pattern is not None:
        if attention_kernel != "softmax":
            raise ValueError(
                f"sparse_pattern is incompatible with attention_kernel={attention_kernel!r}: a "
                "linearized kernel never builds a score matrix, so there is nothing to sparsify.")
        if window_size is not None:
            raise ValueError(
                "sparse_pattern and window_size both restrict which keys a query sees; use "
                "sparse_pattern's 'local' blocks for a windowed pattern rather than combining "
                "the two.")
        from .sparse import normalize_pattern
        sparse_pattern = normalize_pattern(sparse_pattern)
    if tiled_block_size is not None:
        if int(tiled_block_size) < 1:
            raise ValueError(f"tiled_block_size must be >= 1 or None, got {tiled_block_size}")
        if attention_kernel != "softmax" or sparse_pattern is not None:
            raise ValueError(
                "tiled_block_size only applies to the plain softmax path; the linearized kernels "
                "and sparse_pattern already avoid building a score matrix, so there is nothing "
                "to tile.")
        if dropout > 0:
            raise ValueError(
                "tiled_block_size is incompatible with attention dropout: the streaming path "
                "never holds the full attention matrix, so there is nothing to apply a single "
                "consistent dropout mask to.")
        tiled_block_size = int(tiled_block_size)
    if positional_scheme not in ("absolute", "rope", "alibi"):
        raise ValueError(f"Unknown positional_scheme: {positional_scheme!r}. "
                         "Expected 'absolute', 'rope', or 'alibi'.")
    if positional_scheme == "rope" and head_dim % 2 != 0:
        raise ValueError(f"positional_scheme='rope' requires an even head_dim, got {head_dim}")
    Wq, bq = init_weights(embed_dim, embed_dim, method=init_method)
    Wk, bk = init_weights(embed_dim, kv_dim, method=init_method)
    Wv, bv = init_weights(embed_dim, kv_dim, method=init_method)
    Wo, bo = init_weights(embed_dim, embed_dim, method=init_method)
    self.layers.append({
        "type": "multihead_attention", "embed_dim": embed_dim, "num_heads": num_heads,
        "num_kv_heads": num_kv_heads, "head_dim": head_dim, "dropout": dropout,
        "causal": causal, "window_size": window_size, "attention_kernel": attention_kernel,
        "sparse_pattern": sparse_pattern, "tiled_block_size": tiled_block_size,
        "positional_scheme": positional_scheme,
        "Wq": Wq, "bq": bq, "Wk": Wk, "bk": bk, "Wv": Wv, "bv": bv, "Wo": Wo, "bo": bo,
    })
    if omega is not None:
        self.layers[-1]["omega"] = omega
    _set_width(self, embed_dim)


def add_cross_attention(self: Any, kv_source_index: int, embed_dim: Optional[int] = None,
                        num_heads: int = 4, dropout: float = 0.0,
                        init_method: str = "xavier_uniform",
                        num_kv_heads: Optional[int] = None) -> None:
    """Cross-attention, nn/layers.py:404-453: Q from the sequential input,
    K/V from outputs[kv_source_index + 1]."""
    if not (-1 <= kv_source_index < len(self.layers)):
        raise ValueError(
            f"kv_source_index={kv_source_index} is out of range: must be -1 (the raw network "
            f"input) or a valid index into the {len(self.layers)} layer(s) already added "
            "before this cross_attention call.")
    if embed_dim is None:
        embed_dim = _require_width(self, "add_cross_attention")
    if embed_dim % num_heads != 0:
        raise ValueError("embed_dim must be divisible by num_heads")
    head_dim = embed_dim // num_heads
    num_kv_heads = _validate_num_kv_heads(num_heads, num_kv_heads, "add_cross_attention")
    kv_dim = num_kv_heads * head_dim
    Wq, bq = init_weights(embed_dim, embed_dim, method=init_method)
    Wk, bk = init_weights(embed_dim, kv_dim, method=init_method)
    Wv, bv = init_weights(embed_dim, kv_dim, method=init_method)
    Wo, bo = init_weights(embed_dim, embed_dim, method=init_method)
    self.layers.append({
        "type": "cross_attention", "embed_dim": embed_dim, "num_heads": num_heads,
        "num_kv_heads": num_kv_heads, "head_dim": head_dim, "dropout": dropout,
        "kv_source_index": kv_source_index,
        "Wq": Wq, "bq": bq, "Wk": Wk, "bk": bk, "Wv": Wv, "bv": bv, "Wo": Wo, "bo": bo,
    })
    _set_width(self, embed_dim)


# ------------------------------------------------- transformer plumbing
def add_dense(self: Any, n_in: Optional[int] = None, n_out: int = 128, activation: str = "relu",
              init_method: str = "xavier_uniform", use_bias: bool = True,
              activation_params: Optional[Dict[str, Any]] = None) -> None:
    """nn/layers.py:18-29."""
    if n_in is None:
        n_in = _require_width(self, "add_dense")
    w, b = init_weights(n_in, n_out, method=init_method)
    if not use_bias:
        b = np.zeros(n_out, dtype=default_dtype())
    self.layers.append({"type": "dense", "weights": w, "bias": b, "activation": activation,
                        "use_bias": use_bias, "activation_params": activation_params or {}})
    _set_width(self, n_out)


def add_layernorm(self: Any, normalized_shape: Optional[Any] = None,
                  epsilon: float = 1e-5) -> None:
    """nn/layers.py:181-197."""
    if normalized_shape is None:
        normalized_shape = _require_width(self, "add_layernorm")
    n = normalized_shape if isinstance(normalized_shape, int) else math.prod(normalized_shape)
    self.layers.append({"type": "layernorm", "normalized_shape": normalized_shape,
                        "epsilon": epsilon, "gamma": np.ones(n, dtype=default_dtype()),
                        "beta": np.zeros(n, dtype=default_dtype())})


def add_dropout(self: Any, rate: float = 0.5) -> None:
    self.layers.append({"type": "dropout", "rate": rate})


def add_embedding(self: Any, vocab_size: int, embed_dim: int, init_method: str = "normal") -> None:
    """nn/layers.py:199-208."""
    w = init_embedding_weights(vocab_size, embed_dim, method=init_method)
    self.layers.append({"type": "embedding", "weights": w, "vocab_size": vocab_size,
                        "embed_dim": embed_dim})
    _set_width(self, embed_dim)


def add_positional_encoding(self: Any, max_seq_len: int, embed_dim: Optional[int] = None,
                            learnable: bool = True, base: Optional[float] = None) -> None:
    """Learned or sinusoidal table added to the input, nn/transformer_layers.py:59-113."""
    if embed_dim is None:
        if self._last_width is None:
            raise ValueError(
                "Cannot auto-infer embed_dim for add_positional_encoding: no previous layer.")
        embed_dim = self._last_width
    if learnable:
        w = init_embedding_weights(max_seq_len, embed_dim, method="normal")
        self.layers.append({"type": "positional_encoding", "weights": w,
                            "max_seq_len": max_seq_len, "embed_dim": embed_dim,
                            "_is_positional": True, "_pos_type": "learnable"})
    else:
        freq_base = SINUSOIDAL_BASE if base is None else base
        pe = np.zeros((max_seq_len, embed_dim), dtype=default_dtype())
        position = np.arange(max_seq_len).reshape(-1, 1)
        div_term = np.exp(np.arange(0, embed_dim, 2) * -(np.log(freq_base) / embed_dim))
        pe[:, 0::2] = np.sin(position * div_term)
        pe[:, 1::2] = np.cos(position * div_term)
        self.layers.append({"type": "positional_encoding", "pe": pe,
                            "max_seq_len": max_seq_len, "embed_dim": embed_dim,
                            "_is_positional": True, "_pos_type": "sinusoidal"})
    _set_width(self, embed_dim)


def add_residual_start(self: Any) -> None:
    """nn/layers.py:609-622."""
    self._residual_stack.append(len(self.layers))
    self.layers.append({"type": "residual_save",
                        "shape_at_save": [self._last_width, getattr(self, "_last_spatial", None),
                                          getattr(self, "_last_spatial_1d", None)]})


def add_residual_end(self: Any) -> None:
    """nn/layers.py:625-632."""
    if not self._residual_stack:
        raise ValueError("add_residual_end() called without a matching add_residual_start()")
    save_index = self._residual_stack.pop()
    self.layers.append({"type": "residual_add", "save_index": save_index})
    saved = self.layers[save_index].get("shape_at_save")
    if saved is not None:
        self._last_width = saved[0]


def add_transformer_block(self: Any, embed_dim: Optional[int] = None, num_heads: int = 4,
                          mlp_ratio: float = 4.0, dropout: float = 0.0,
                          activation: str = "swish", causal: bool = False,
                          positional_scheme: str = "absolute",
                          num_kv_heads: Optional[int] = None,
                          window_size: Optional[int] = None,
                          attention_kernel: str = "softmax",
                          num_features: Optional[int] = None,
                          sparse_pattern: Optional[Any] = None,
                          tiled_block_size: Optional[int] = None) -> None:
    """Pre-norm block LN -> MHA -> residual -> LN -> MLP -> residual,
    nn/transformer_layers.py:13-57."""
    if embed_dim is None:
        if self._last_width is None:
            raise ValueError(
                "Cannot auto-infer embed_dim for add_transformer_block: no previous layer.")
        embed_dim = self._last_width
    add_residual_start(self)
    add_layernorm(self, (embed_dim,))
    add_multihead_attention(self, embed_dim, num_heads, dropout, causal=causal,
                            positional_scheme=positional_scheme, num_kv_heads=num_kv_heads,
                            window_size=window_size, attention_kernel=attention_kernel,
                            num_features=num_features, sparse_pattern=sparse_pattern,
                            tiled_block_size=tiled_block_size)
    add_residual_end(self)
    add_residual_start(self)
    add_layernorm(self, (embed_dim,))
    hidden = int(embed_dim * mlp_ratio)
    add_dense(self, embed_dim, hidden, activation=activation, init_method="xavier_uniform")
    add_dense(self, hidden, embed_dim, activation="linear", init_method="xavier_uniform")
    if dropout > 0:
        add_dropout(self, dropout)
    add_residual_end(self)


BUILDERS = {
    "add_multihead_attention": add_multihead_attention,
    "add_cross_attention": add_cross_attention,
    "add_transformer_block": add_transformer_block,
    "add_dense": add_dense,
    "add_layernorm": add_layernorm,
    "add_dropout": add_dropout,
    "add_embedding": add_embedding,
    "add_positional_encoding": add_positional_encoding,
    "add_residual_start": add_residual_start,
    "add_residual_end": add_residual_end,
}
