"""A char-level tokenizer with the reference Tokenizer's interface, rebuilt
from the vocabulary stored in tests/golden/textgen.npz (no reference import)."""
import json

import numpy as np


class CharTokenizer:
    pad_token, start_token, end_token, oov_token = "<PAD>", "<START>", "<END>", "<OOV>"

    def __init__(self, word_to_idx):
        self.word_to_idx = dict(word_to_idx)
        self.idx_to_word = {i: w for w, i in self.word_to_idx.items()}
        self.fitted = True

    def encode(self, text, max_length=None, add_special_tokens=True):
        ids = [self.word_to_idx[self.start_token]] if add_special_tokens else []
        ids += [self.word_to_idx.get(c, self.word_to_idx[self.oov_token]) for c in text]
        if add_special_tokens:
            ids.append(self.word_to_idx[self.end_token])
        return np.array(ids, dtype=np.int64)

    def decode(self, indices, skip_special=True):
        special = {self.pad_token, self.start_token, self.end_token}
        out = []
        for i in indices:
            tok = self.idx_to_word.get(int(i), self.oov_token)
            if skip_special and tok in special:
                continue
            out.append(tok)
        return "".join(out)


def load(golden_dir):
    data = np.load(golden_dir / "textgen.npz")
    return data, CharTokenizer(json.loads(str(data["vocab"])))


PROMPTS = ["the cache", "a small", "keys and", "values"]
CORPUS0 = "attention reads keys and values; the cache keeps them close."
