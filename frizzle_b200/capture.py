"""The capture store: its layout and a reader over one sequence's store.

``layout`` restates ``capture::layout`` (src/core/capture/capture.cpp:31-73):
region 1 holds every layer's neurons, in layer order; region 2, a layer at a
time, its residual, attention addition and feed-forward addition (the
embedding width each), its query (query heads x head dimension), its
attention weights (query heads x keys, keys = min(window, trained
context)), its statistics (m then l, a head) and its readout (64 pairs of
logit bits and token), each slot after the last, in 32-bit words.

``Capture`` reads one sequence's store the way ``capture::Reader``
(src/core/capture/reader.h:90-113) hands it to the page: per layer, the
vectors, the weights over the keys the captured row read, and the readout as
(logit, token) pairs, best first.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

READOUT_PAIRS = 64                 # residency::kCandidates
READOUT_WORDS = 2 * READOUT_PAIRS  # capture::kReadoutWords
SLOTS = ("neurons", "residual", "attention_added", "mlp_added", "query", "weights", "stats", "readout")


@dataclass(frozen=True)
class LayerSlots:
    """One layer's slots, (first word, width) each, and its attention."""
    neurons: tuple
    residual: tuple
    attention_added: tuple
    mlp_added: tuple
    query: tuple
    weights: tuple
    stats: tuple
    readout: tuple
    keys: int
    query_heads: int
    window: int
    full_attention: bool


@dataclass(frozen=True)
class Layout:
    layers: tuple
    neuron_words: int
    words: int


def _window(shape, layer: int) -> int:
    if shape.window == 0 or layer % shape.pattern == shape.pattern - 1:
        return shape.context
    return shape.window


def layout(shape) -> Layout:
    """Where every slot lies, for a shape with layers, hidden, ffn, heads,
    head_dim, window, pattern and context (the trained context)."""
    at = 0

    def take(width: int):
        nonlocal at
        slot = (at, width)
        at += width
        return slot

    neurons = [take(shape.ffn) for _ in range(shape.layers)]
    neuron_words = at
    layers = []
    for l in range(shape.layers):
        window = _window(shape, l)
        keys = min(window, shape.context)
        residual = take(shape.hidden)
        attention_added = take(shape.hidden)
        mlp_added = take(shape.hidden)
        query = take(shape.heads * shape.head_dim)
        weights = take(shape.heads * keys)
        stats = take(2 * shape.heads)
        readout = take(READOUT_WORDS)
        layers.append(LayerSlots(neurons[l], residual, attention_added, mlp_added, query, weights, stats, readout,
                                 keys, shape.heads, window, window >= shape.context))
    if at > 0xFFFFFFFF:
        raise ValueError("a capture store past 2^32 words")
    return Layout(tuple(layers), neuron_words, at)


class Capture:
    """One sequence's capture store (float32 words) read through its layout."""

    def __init__(self, store: np.ndarray, lay: Layout, head_dim: int):
        if store.size < lay.words:
            raise ValueError("the store is shorter than the layout")
        self.store = np.ascontiguousarray(store, dtype=np.float32)
        self.layout = lay
        self.head_dim = head_dim

    def _slot(self, layer: int, name: str) -> np.ndarray:
        first, width = getattr(self.layout.layers[layer], name)
        return self.store[first:first + width]

    def neurons(self, layer: int) -> np.ndarray:
        return self._slot(layer, "neurons")

    def residual(self, layer: int) -> np.ndarray:
        return self._slot(layer, "residual")

    def attention_added(self, layer: int) -> np.ndarray:
        return self._slot(layer, "attention_added")

    def mlp_added(self, layer: int) -> np.ndarray:
        return self._slot(layer, "mlp_added")

    def query(self, layer: int) -> np.ndarray:
        """[query heads][head dimension], after QK-norm and RoPE."""
        s = self.layout.layers[layer]
        return self._slot(layer, "query").reshape(s.query_heads, self.head_dim)

    def weights(self, layer: int) -> np.ndarray:
        """[query heads][keys]: key i is position earliest + i; zeros past the keys read."""
        s = self.layout.layers[layer]
        return self._slot(layer, "weights").reshape(s.query_heads, s.keys)

    def stats(self, layer: int) -> np.ndarray:
        """[query heads][2]: the softmax maximum m and sum l, in log2 units."""
        s = self.layout.layers[layer]
        return self._slot(layer, "stats").reshape(s.query_heads, 2)

    def readout(self, layer: int):
        """(logits float32[64], tokens uint32[64]), best first."""
        words = self._slot(layer, "readout").view(np.uint32).reshape(READOUT_PAIRS, 2)
        return words[:, 0].copy().view(np.float32), words[:, 1].copy()

    def activations(self) -> np.ndarray:
        """Every layer's vectors (neurons, residual, additions, query) in one array."""
        parts = []
        for l in range(len(self.layout.layers)):
            parts += [self.neurons(l), self.residual(l), self.attention_added(l), self.mlp_added(l),
                      self.query(l).ravel()]
        return np.concatenate(parts)
