"""Install the B200 decoder on an engine object of the reference package.

The reference's seam for its CUDA path is one attribute: ``LFM25Engine._cuda_decoder``, set by
``LFM25Engine.enable_cuda_graphs`` (src/climbing_gym/inference/lfm25_engine.py:980-1002) and consulted by
``generate`` (:749-750), ``sync_from_model`` (:573-577), ``release_inference_buffers`` (:580-591) and
``disable_cuda_graphs`` (:999-1002). ``install`` puts this package's decoder there:

* the reference engine's packed weight tensors (``LFM25PackedWeights``, :88-223 - same field names and
  layouts as this package's) are adopted without a copy, so the reference's in-place weight sync
  (``copy_from_model_`` + ``refresh_weights``) keeps working and both sides see one set of buffers;
* ``reference_engine.generate`` then reaches ``B200Decoder.generate`` through the reference's own method;
* ``reference_engine.generation_session`` is rebound to this package's session (the reference's session class
  drives its decoder's dense cache directly, :120-176 of lfm25_session.py, which the paged cache replaces).

What the decoder needs beyond the reference engine's attributes - the paged cache factory, packed varlen
prefill, RoPE tables in its own layout - lives in this package's ``LFM25Engine``; the bridge builds one
around the adopted weights and keeps it on the decoder (``decoder.engine``).
"""
from __future__ import annotations

from typing import Any

from .engine import LFM25Engine
from .weights import (LFM25AttentionWeights, LFM25ConvWeights, LFM25LayerWeights, LFM25PackedWeights, coerce_config)


def adopt_weights(reference_weights: Any) -> LFM25PackedWeights:
    """This package's view of a reference ``LFM25PackedWeights``: the same tensors, no copies."""
    layers = []
    for layer in reference_weights.layers:
        attention = conv = None
        if layer.attention is not None:
            a = layer.attention
            attention = LFM25AttentionWeights(a.qkv_weight, a.out_weight, a.q_norm_weight, a.k_norm_weight, a.cache_index)
        if layer.conv is not None:
            c = layer.conv
            conv = LFM25ConvWeights(c.in_weight, c.conv_weight, c.out_weight, c.cache_index)
        layers.append(LFM25LayerWeights(layer.operator_norm_weight, layer.ffn_norm_weight, layer.w13_weight,
                                        layer.w2_weight, attention, conv))
    return LFM25PackedWeights(coerce_config(reference_weights.config), reference_weights.embed_tokens,
                              reference_weights.embedding_norm_weight, reference_weights.lm_head_weight, tuple(layers),
                              reference_weights.device, reference_weights.dtype)


class _BridgedEngine(LFM25Engine):
    """This package's engine over adopted weights; the policy version is the reference engine's."""

    def __init__(self, reference_engine: Any):
        self._reference = reference_engine
        super().__init__(adopt_weights(reference_engine.weights), max_model_len=int(reference_engine.max_model_len))

    @property
    def policy_version(self) -> int:
        return int(self._reference.policy_version)

    @policy_version.setter
    def policy_version(self, value: int) -> None:
        pass  # owned by the reference engine (its sync_from_model increments it)


def install(reference_engine: Any, **graph_options):
    """``reference_engine.enable_cuda_graphs(**graph_options)`` with this package's decoder. Returns the
    decoder now stored in ``reference_engine._cuda_decoder``."""
    current = getattr(reference_engine, "_cuda_decoder", None)
    if current is not None and current._active_session is not None:
        raise RuntimeError("Close the native generation session before reconfiguring CUDA graphs")
    engine = _BridgedEngine(reference_engine)
    engine.enable_cuda_graphs(**graph_options)
    decoder = engine._cuda_decoder
    reference_engine._cuda_decoder = decoder
    reference_engine.generation_session = engine.generation_session
    return decoder


def uninstall(reference_engine: Any) -> None:
    """Undo ``install``: clear the decoder and give ``generation_session`` back to the reference class."""
    decoder = getattr(reference_engine, "_cuda_decoder", None)
    if decoder is not None:
        decoder.clear()
    reference_engine._cuda_decoder = None
    reference_engine.__dict__.pop("generation_session", None)
