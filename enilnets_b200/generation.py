"""Autoregressive text generation on the B200 attention path.

This is the inference half of the reference's `TextGenerator`
(generative/text_generation.py:10-400). The constructor builds the same
GPT-style stack with this package's builders, in the same RNG order, so a
given seed gives the reference's weights. The decode loops are built the way
the reference builds them:
  * sampled / greedy generation, primed in one cached step, then one token a
    step (text_generation.py:136-198);
  * beam search over one shared cache, reordered by parent beam after every
    prune (text_generation.py:200-313);
  * batched generation, with prompts grouped by token length and each group
    decoded as one exact batch (text_generation.py:315-381);
  * perplexity (text_generation.py:383-398).
They run on `cached_forward_step` / `KVCache` of `enilnets_b200.kvcache`,
where K/V stay on the device, each step appends with K3 and attends with K2.
Beam pruning gathers the cache rows on the device (`kv_gather_kernel`).

Training (`train_step`, `Train`) belongs to the reference; the B200 path is
inference only, and those methods raise.
"""
from __future__ import annotations

from typing import Any, List, Optional, Sequence, Tuple

import numpy as np

from .backend import default_dtype
from .kvcache import KVCache, cached_forward_step
from .network import AttentionNet

_TOKENIZER_API = ("encode", "decode", "word_to_idx", "fitted", "pad_token", "start_token",
                  "end_token", "oov_token")


# ------------------------------------------------------------- sampling
def top_k_renormalize(probs: np.ndarray, k: int) -> np.ndarray:
    """Keep the k largest entries of one distribution and renormalise
    (generative/sampling.py:108-120: the kept set is argpartition's)."""
    k = min(int(k), probs.shape[-1])
    kept = np.argpartition(probs, -k)[-k:]
    out = np.zeros_like(probs)
    out[kept] = probs[kept]
    return out / out.sum()


def nucleus_renormalize(probs: np.ndarray, top_p: float) -> np.ndarray:
    """Per row of (batch, vocab): keep the smallest set of the largest
    entries whose mass reaches top_p (the entry that crosses it included) and
    renormalise (generative/sampling.py:57-82)."""
    order = np.argsort(probs, axis=-1)[..., ::-1]
    ranked = np.take_along_axis(probs, order, axis=-1)
    before = np.cumsum(ranked, axis=-1) - ranked  # mass ahead of each entry
    ranked = np.where(before < top_p, ranked, 0.0)
    out = np.zeros_like(probs)
    np.put_along_axis(out, order, ranked, axis=-1)
    return out / out.sum(axis=-1, keepdims=True)


def sample_token(probs: Any, temperature: float = 1.0, top_p: Optional[float] = None,
                 top_k: Optional[int] = None, greedy: bool = False) -> int:
    """One token id from a next-token distribution, with the reference's
    order of operations (text_generation.py:118-134): argmax when greedy,
    else temperature, then top-k, then top-p, then one draw from NumPy's
    global RNG."""
    if greedy:
        return int(np.argmax(probs))
    p = np.array(probs, dtype=default_dtype())
    if temperature != 1.0:
        p = np.power(np.maximum(p, 1e-12), 1.0 / temperature)
        p = p / p.sum()
    if top_k is not None:
        p = top_k_renormalize(p, top_k)
    if top_p is not None:
        p = nucleus_renormalize(p.reshape(1, -1), top_p)[0]
    return int(np.random.choice(len(p), size=1, p=p)[0])


def sliding_windows(ids: np.ndarray, width: int, stride: int = 1) -> Tuple[np.ndarray, np.ndarray]:
    """(X, y) next-token windows of `width` tokens, y = X shifted by one
    (text/text_utils.py:151-165)."""
    if width >= len(ids):
        raise ValueError(f"window_size={width} must be < len(data)={len(ids)}")
    starts = range(0, len(ids) - width, stride)
    win = np.stack([ids[s:s + width + 1] for s in starts])
    return win[:, :-1], win[:, 1:]


# ------------------------------------------------------------ generator
class TextGenerator:
    """TextGenerator(tokenizer, embed_dim=64, num_heads=4, num_layers=2,
    mlp_ratio=4.0, dropout=0.0, activation="gelu", max_seq_len=128, ...)
    with the reference's inference methods. `tokenizer` follows the
    reference's Tokenizer interface (duck-typed)."""

    def __init__(self, tokenizer: Any, embed_dim: int = 64, num_heads: int = 4,
                 num_layers: int = 2, mlp_ratio: float = 4.0, dropout: float = 0.0,
                 activation: str = "gelu", max_seq_len: int = 128, learning_rate: float = 3e-4,
                 optimizer: str = "adam", l2_lambda: float = 0.0) -> None:
        missing = [name for name in _TOKENIZER_API if not hasattr(tokenizer, name)]
        if missing:
            raise ValueError(
                f"tokenizer is missing {missing}; it needs the same interface as "
                "Enilnets.Tokenizer or Enilnets.BPETokenizer")
        if not tokenizer.fitted:
            raise ValueError("tokenizer must be fitted -- call fit(texts) first")
        self.tokenizer = tokenizer
        self.vocab_size = len(tokenizer.word_to_idx)
        self.max_seq_len = max_seq_len
        self.embed_dim = embed_dim
        # learning_rate / optimizer / l2_lambda configure the reference's
        # training, which this path does not run; kept for signature parity.
        net = AttentionNet()
        net.add_embedding(self.vocab_size, embed_dim)
        net.add_positional_encoding(max_seq_len, embed_dim, learnable=False)
        for _ in range(num_layers):
            net.add_transformer_block(embed_dim, num_heads, mlp_ratio=mlp_ratio, dropout=dropout,
                                      activation=activation, causal=True)
        net.add_layernorm()
        net.add_dense(None, self.vocab_size, activation="softmax")
        self.network = net

    @classmethod
    def from_layers(cls, tokenizer: Any, layers: Sequence[dict], max_seq_len: int) -> "TextGenerator":
        """Wrap a stack of layer dicts (e.g. a trained reference model's
        `network.layers`) without drawing new weights."""
        self = cls.__new__(cls)
        self.tokenizer = tokenizer
        self.vocab_size = len(tokenizer.word_to_idx)
        self.max_seq_len = max_seq_len
        self.network = AttentionNet()
        self.network.layers = list(layers)
        self.embed_dim = self.network.layers[0].get("embed_dim")
        return self

    # -- training belongs to the reference
    def train_step(self, *args: Any, **kwargs: Any) -> float:
        raise NotImplementedError("the B200 attention path is inference-only; train with the "
                                  "reference TextGenerator and load its layers with from_layers")

    def Train(self, *args: Any, **kwargs: Any) -> List[float]:
        return self.train_step()

    # -- helpers
    def _id(self, token: str) -> int:
        return self.tokenizer.word_to_idx[token]

    def _prompt_ids(self, prompt: str) -> List[int]:
        ids = [self._id(self.tokenizer.start_token)]
        if prompt:
            ids += self.tokenizer.encode(prompt, add_special_tokens=False).tolist()
        return ids

    def _sample_token(self, probs: Any, temperature: float = 1.0, top_p: Optional[float] = None,
                      top_k: Optional[int] = None, greedy: bool = False) -> int:
        return sample_token(probs, temperature, top_p, top_k, greedy)

    # -- generation
    def generate_ids(self, prompt: str = "", max_new_tokens: int = 100, temperature: float = 1.0,
                     top_p: Optional[float] = None, top_k: Optional[int] = None,
                     greedy: bool = False, use_cache: bool = True) -> List[int]:
        """Token ids of `generate` (prompt included, special tokens kept)."""
        end_id = self._id(self.tokenizer.end_token)
        ids = self._prompt_ids(prompt)
        if not use_cache:
            for _ in range(max_new_tokens):
                context = np.array([ids[-self.max_seq_len:]], dtype=np.int64)
                probs = self.network.Forward(context, training=False)[0, -1]
                nxt = self._sample_token(probs, temperature, top_p, top_k, greedy)
                if nxt == end_id:
                    break
                ids.append(nxt)
            return ids
        # Prime with the (truncated) prompt in one step, then one token a step.
        cache = KVCache()
        probs = cached_forward_step(self.network, [ids[-self.max_seq_len:]], cache)[0, -1]
        for _ in range(max_new_tokens):
            nxt = self._sample_token(probs, temperature, top_p, top_k, greedy)
            if nxt == end_id:
                break
            ids.append(nxt)
            if cache.position >= self.max_seq_len:
                break
            probs = cached_forward_step(self.network, [[nxt]], cache)[0, -1]
        return ids

    def generate(self, prompt: str = "", max_new_tokens: int = 100, temperature: float = 1.0,
                 top_p: Optional[float] = None, top_k: Optional[int] = None,
                 greedy: bool = False, use_cache: bool = True) -> str:
        ids = self.generate_ids(prompt, max_new_tokens, temperature, top_p, top_k, greedy,
                                use_cache)
        return self.tokenizer.decode(ids, skip_special=True)

    def beam_ids(self, prompt: str = "", beam_width: int = 5, max_new_tokens: int = 50,
                 length_penalty: float = 1.0, top_k: Optional[int] = None,
                 use_cache: bool = True) -> List[int]:
        """Token ids of `generate_beam`'s best beam."""
        end_id = self._id(self.tokenizer.end_token)
        init = self._prompt_ids(prompt)
        expand = beam_width if top_k is None else int(top_k)
        if expand < 1:
            raise ValueError(f"top_k must be >= 1 (or None), got {top_k}")
        if beam_width < 1:
            raise ValueError(f"beam_width must be >= 1, got {beam_width}")

        def norm(logprob: float, length: int) -> float:
            return logprob / (length ** length_penalty)

        if not use_cache:
            beams = [(init, 0.0, False)]
            for _ in range(max_new_tokens):
                live = [(ids, lp) for ids, lp, done in beams if not done]
                if not live:
                    break
                ctx = np.array([ids[-self.max_seq_len:] for ids, _ in live], dtype=np.int64)
                rows = np.clip(self.network.Forward(ctx, training=False)[:, -1, :], 1e-12, 1.0)
                cand = [(ids, lp, True) for ids, lp, done in beams if done]
                for (ids, lp), row in zip(live, rows):
                    for tok in np.argsort(-row)[:expand]:
                        tok = int(tok)
                        cand.append((ids + [tok], lp + float(np.log(row[tok])), tok == end_id))
                cand.sort(key=lambda c: norm(c[1], len(c[0])), reverse=True)
                beams = cand[:beam_width]
            return max(beams, key=lambda c: norm(c[1], len(c[0])))[0] if beams else init

        # One shared cache that widens and narrows with the surviving beams;
        # a finished beam stays pinned to the end token with its score.
        cache = KVCache()
        rows = cached_forward_step(self.network, [init[-self.max_seq_len:]], cache)[:, -1, :]
        seqs, lps, done = [list(init)], [0.0], [False]
        for _ in range(max_new_tokens):
            if all(done) or cache.position >= self.max_seq_len:
                break
            cand = []  # (score, parent, token, logprob, done)
            for b, seq in enumerate(seqs):
                if done[b]:
                    cand.append((norm(lps[b], len(seq)), b, end_id, lps[b], True))
                    continue
                row = np.clip(rows[b], 1e-12, 1.0)
                for tok in np.argsort(-row)[:expand]:
                    tok = int(tok)
                    lp = lps[b] + float(np.log(row[tok]))
                    cand.append((norm(lp, len(seq) + 1), b, tok, lp, tok == end_id))
            cand.sort(key=lambda c: c[0], reverse=True)
            kept = cand[:beam_width]
            cache.reorder([c[1] for c in kept])
            seqs = [seqs[c[1]] + [c[2]] for c in kept]
            lps = [c[3] for c in kept]
            done = [c[4] for c in kept]
            rows = cached_forward_step(self.network, [[c[2]] for c in kept], cache)[:, -1, :]
        best = max(range(len(seqs)), key=lambda b: norm(lps[b], len(seqs[b])))
        return seqs[best]

    def generate_beam(self, prompt: str = "", beam_width: int = 5, max_new_tokens: int = 50,
                      length_penalty: float = 1.0, top_k: Optional[int] = None,
                      use_cache: bool = True) -> str:
        ids = self.beam_ids(prompt, beam_width, max_new_tokens, length_penalty, top_k, use_cache)
        return self.tokenizer.decode(ids, skip_special=True)

    def batch_ids(self, prompts: List[str], max_new_tokens: int = 100, temperature: float = 1.0,
                  top_p: Optional[float] = None, top_k: Optional[int] = None,
                  greedy: bool = False) -> List[List[int]]:
        """Token ids of `generate_batch`, one list per prompt in order.
        Prompts of equal token length share one exact batch and cache (no
        padding: the nn/ attention has no padding mask)."""
        end_id = self._id(self.tokenizer.end_token)
        encoded = [self._prompt_ids(p)[-self.max_seq_len:] for p in prompts]
        groups: dict = {}
        for i, ids in enumerate(encoded):
            groups.setdefault(len(ids), []).append(i)
        out: List[Optional[List[int]]] = [None] * len(prompts)
        for members in groups.values():
            cache = KVCache()
            batch = np.array([encoded[i] for i in members], dtype=np.int64)
            rows = cached_forward_step(self.network, batch, cache)[:, -1, :]
            seqs = [list(encoded[i]) for i in members]
            done = [False] * len(members)
            for _ in range(max_new_tokens):
                if all(done) or cache.position >= self.max_seq_len:
                    break
                step = []
                for b in range(len(members)):
                    if done[b]:
                        step.append(end_id)
                        continue
                    tok = self._sample_token(rows[b], temperature, top_p, top_k, greedy)
                    if tok == end_id:
                        done[b] = True
                    else:
                        seqs[b].append(tok)
                    step.append(tok)
                rows = cached_forward_step(self.network, [[t] for t in step], cache)[:, -1, :]
            for i, seq in zip(members, seqs):
                out[i] = seq
        return [o for o in out]

    def generate_batch(self, prompts: List[str], max_new_tokens: int = 100,
                       temperature: float = 1.0, top_p: Optional[float] = None,
                       top_k: Optional[int] = None, greedy: bool = False) -> List[str]:
        if not prompts:
            return []
        return [self.tokenizer.decode(ids, skip_special=True)
                for ids in self.batch_ids(prompts, max_new_tokens, temperature, top_p, top_k,
                                          greedy)]

    def perplexity(self, text: str) -> float:
        """exp(mean next-token cross-entropy) over `text`, in non-overlapping
        windows of up to max_seq_len - 1 tokens (text_generation.py:383-398)."""
        ids = self.tokenizer.encode(text, add_special_tokens=True).tolist()
        if len(ids) < 2:
            raise ValueError("Need at least 2 tokens (after tokenization) to compute perplexity.")
        width = min(self.max_seq_len - 1, len(ids) - 1)
        X, y = sliding_windows(np.array(ids, dtype=np.int64), width, stride=width)
        probs = np.clip(self.network.Forward(X, training=False), 1e-12, 1.0)
        picked = np.take_along_axis(probs, y[..., None], axis=-1)[..., 0]
        return float(np.exp(-np.mean(np.log(picked))))
