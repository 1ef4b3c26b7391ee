"""ASCII stop strings as a token-level automaton, so stop matching never decodes text on the hot path.

Table format (shared with the sampler kernel's bookkeeping and with the reference,
src/climbing_gym/inference/text_stops.py:6-45): ``table[state, token] = next_state + 65536 * matched``
as int32 ``[states, vocab]``. A state is a proper prefix of some stop string that the generated text
currently ends with (state 0 = empty prefix); ``matched`` is set when appending the token's text
completes any stop string.
"""
from __future__ import annotations

import numpy as np
import torch


def trim_after_stop(text: str, stops) -> str:
    """Cut ``text`` right after the earliest-ending completed stop string (display only: the
    sampled token that contained the stop, and its log-prob, stay in the rollout)."""
    cut = None
    for stop in stops:
        if not stop:
            continue
        at = text.find(stop)
        if at >= 0:
            end = at + len(stop)
            cut = end if cut is None else min(cut, end)
    return text if cut is None else text[:cut]


def build_stop_table(tokenizer, stops, *, vocab_size=None) -> torch.Tensor:
    if any(not s or not s.isascii() for s in stops):
        raise ValueError("Native text stops must be nonempty ASCII strings")
    states = sorted({""} | {s[:i] for s in stops for i in range(1, len(s))}, key=len)
    if len(states) >= 65536:
        raise ValueError("Too many stop-prefix states")
    n_tok = len(tokenizer)
    vocab = n_tok if vocab_size is None else int(vocab_size)
    if vocab < n_tok:
        raise ValueError("Model vocabulary must cover the tokenizer vocabulary")
    pieces = [tokenizer.decode([i], skip_special_tokens=False, clean_up_tokenization_spaces=False)
              for i in range(n_tok)]
    # ids past the tokenizer (padded output head) decode to nothing and keep the current state
    pieces += [""] * (vocab - n_tok)
    by_length = sorted(range(len(states)), key=lambda i: -len(states[i]))
    table = np.zeros((len(states), vocab), dtype=np.int32)
    for index, prefix in enumerate(states):
        for token, piece in enumerate(pieces):
            text = prefix + piece
            longest = next(i for i in by_length if text.endswith(states[i]))
            table[index, token] = longest + (65536 if any(s in text for s in stops) else 0)
    return torch.from_numpy(table)


def advance_text_stops(table, states, tokens, reasons):
    value = table[states, tokens].long()
    return value & 65535, torch.where((reasons == 0) & (value >= 65536), 2, reasons)


def build_token_sequence_table(sequences, vocab_size: int) -> torch.Tensor:
    """The same table format for stop TOKEN sequences (``LFM25SamplingConfig.stop_token_sequences``):
    generation stops when the generated ids end with any of the sequences, the match the reference
    makes with ``apply_sequence_stops`` on the token history
    (src/climbing_gym/inference/lfm25_engine.py:1620-1626). States are the proper prefixes of the
    sequences (an Aho-Corasick automaton over token ids); only ids that occur in a sequence ever leave
    state 0, so the table is filled column by column for those ids alone."""
    patterns = [tuple(int(t) for t in s) for s in sequences]
    if any(not p for p in patterns):
        raise ValueError("Stop token sequences must be nonempty")
    if any(not 0 <= t < vocab_size for p in patterns for t in p):
        raise ValueError("Stop token outside the model vocabulary")
    states = sorted({()} | {p[:i] for p in patterns for i in range(1, len(p))}, key=lambda s: (len(s), s))
    if len(states) >= 65536:
        raise ValueError("Too many stop-prefix states")
    index = {state: i for i, state in enumerate(states)}
    table = np.zeros((len(states), int(vocab_size)), dtype=np.int32)
    for state in states:
        for token in {t for p in patterns for t in p}:
            history = state + (token,)
            matched = any(history[-len(p):] == p for p in patterns if len(p) <= len(history))
            longest = next(history[cut:] for cut in range(len(history) + 1) if history[cut:] in index)
            table[index[state], token] = index[longest] + (65536 if matched else 0)
    return torch.from_numpy(table)


def product_stop_table(first: torch.Tensor, second: torch.Tensor) -> torch.Tensor:
    """Two stop automata advanced in lock step as one table: state ``a * states(second) + b``, matched
    when either matches. This is what a request with both a ``stop_table`` and ``stop_token_sequences``
    means in the reference's loop, which advances the text table and then tests the token suffixes
    (src/climbing_gym/inference/lfm25_cuda.py:343-347)."""
    if first.ndim != 2 or second.ndim != 2 or first.size(1) != second.size(1):
        raise ValueError("stop tables must be [states, vocab] over the same vocabulary")
    n_first, n_second = first.size(0), second.size(0)
    if n_first * n_second >= 65536:
        raise ValueError("Too many stop-prefix states")
    second = second.to(first.device)
    a, b = first.to(torch.int64)[:, None, :], second.to(torch.int64)[None, :, :]
    state = (a & 65535) * n_second + (b & 65535)
    matched = ((a >> 16) | (b >> 16)) != 0
    return (state + matched * 65536).reshape(n_first * n_second, -1).to(torch.int32)
