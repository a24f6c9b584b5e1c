"""TextGenerator on the B200 path, host side: the constructor draws exactly
the reference's weights (SHA-256 of every array, in layer order), validates
the tokenizer like the reference, and the host sampling helpers follow the
reference's top-k / nucleus rules."""
import json

import numpy as np
import pytest

import enilnets_b200 as enl
from enilnets_b200 import generation
from tests.textgen_util import load


def test_textgen_weights_match_reference_digests(golden_dir):
    import hashlib
    data, tok = load(golden_dir)
    enl.use_float64(True)
    try:
        enl.set_seed(42)
        gen = generation.TextGenerator(tok, embed_dim=32, num_heads=4, num_layers=2,
                                       max_seq_len=48)
        digests = [hashlib.sha256(np.ascontiguousarray(layer[k]).tobytes()).hexdigest()
                   for layer in gen.network.layers for k in sorted(layer)
                   if isinstance(layer[k], np.ndarray)]
    finally:
        enl.use_float64(False)
    assert digests == json.loads(str(data["digests"]))


def test_tokenizer_validation(golden_dir):
    _, tok = load(golden_dir)
    class Missing:
        fitted = True
    with pytest.raises(ValueError, match="missing"):
        generation.TextGenerator(Missing())
    tok.fitted = False
    with pytest.raises(ValueError, match="fitted"):
        generation.TextGenerator(tok)


def test_training_is_refused(golden_dir):
    _, tok = load(golden_dir)
    gen = generation.TextGenerator(tok, embed_dim=16, num_heads=2, num_layers=1, max_seq_len=16)
    with pytest.raises(NotImplementedError, match="inference-only"):
        gen.Train(["abc"])


def test_sampling_helpers():
    p = np.array([0.1, 0.4, 0.2, 0.3])
    np.testing.assert_allclose(generation.top_k_renormalize(p, 2), [0, 4 / 7, 0, 3 / 7])
    # nucleus: keep the smallest top set whose mass reaches top_p, the
    # crossing entry included (0.4 + 0.3 >= 0.5)
    np.testing.assert_allclose(generation.nucleus_renormalize(p[None], 0.5)[0],
                               [0, 4 / 7, 0, 3 / 7])
    np.testing.assert_allclose(generation.nucleus_renormalize(p[None], 0.35)[0], [0, 1, 0, 0])
    assert generation.sample_token(p, greedy=True) == 1
    X, y = generation.sliding_windows(np.arange(7), 3, stride=3)
    assert X.tolist() == [[0, 1, 2], [3, 4, 5]] and y.tolist() == [[1, 2, 3], [4, 5, 6]]
