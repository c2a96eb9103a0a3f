"""Seeded synthetic inputs for the drafter benchmarks and parity tests.

The reference measures draft quality on Spec-Bench replays, which are not
available here; these generators produce token streams with the shapes,
vocabularies and repetition structure of the five benchmark configurations:
bounded Zipf draws mixed with copies of earlier spans of the same stream
(the structure that makes suffix drafting work).

All generators use ``numpy.random.default_rng(seed)`` and return host numpy
arrays; callers move them to the device.
"""

from __future__ import annotations

import numpy as np


class Zipf:
    """Bounded Zipf(s) over ``vocab`` ids: P(id = r-1) ∝ r^-s, r in 1..V,
    sampled by inverse CDF."""

    def __init__(self, s: float, vocab: int):
        w = np.arange(1, vocab + 1, dtype=np.float64) ** (-s)
        self.cdf = np.cumsum(w) / w.sum()
        self.vocab = vocab

    def draw(self, rng: np.random.Generator, n) -> np.ndarray:
        u = rng.random(n)
        return np.minimum(np.searchsorted(self.cdf, u, side="right"),
                          self.vocab - 1).astype(np.int32)


def copy_stream(rng: np.random.Generator, n: int, zipf: Zipf,
                p_copy: float, span_lo: int, span_hi: int,
                fresh_len: int | tuple[int, int] = 64) -> np.ndarray:
    """A stream of segments: with probability ``p_copy`` a segment copies an
    earlier span (length U[span_lo, span_hi]) of the same stream, otherwise
    it is ``fresh_len`` (an int or a U[lo, hi] range) fresh Zipf draws."""
    out = np.empty(n, dtype=np.int32)
    pos = 0
    while pos < n:
        if pos >= span_lo and rng.random() < p_copy:
            ln = int(rng.integers(span_lo, span_hi + 1))
            ln = min(ln, pos)
            src = int(rng.integers(0, pos - ln + 1))
            m = min(ln, n - pos)
            out[pos:pos + m] = out[src:src + m]
        else:
            if isinstance(fresh_len, tuple):
                ln = int(rng.integers(fresh_len[0], fresh_len[1] + 1))
            else:
                ln = fresh_len
            m = min(ln, n - pos)
            out[pos:pos + m] = zipf.draw(rng, m)
        pos += m
    return out


def sampled_tokens(rng: np.random.Generator, b: int, t: int,
                   zipf: Zipf) -> np.ndarray:
    """[B, T] int32 sampled ids: U[1, T] accepted per row, -1 after."""
    cnt = rng.integers(1, t + 1, size=b)
    tok = zipf.draw(rng, (b, t))
    tok[np.arange(t)[None, :] >= cnt[:, None]] = -1
    return tok.astype(np.int32)


def local_config(seed: int, b: int, s: int, vocab: int, p_copy: float,
                 span: tuple[int, int], q_range: tuple[int, int],
                 steps: int = 1, t: int = 5, zipf_s: float = 1.1) -> dict:
    """Rows of copy/Zipf segments plus ``steps`` batches of sampled ids."""
    rng = np.random.default_rng(seed)
    z = Zipf(zipf_s, vocab)
    tok = np.stack([copy_stream(rng, s, z, p_copy, span[0], span[1])
                    for _ in range(b)])
    q = rng.integers(q_range[0], q_range[1] + 1, size=b).astype(np.int32)
    sampled = np.stack([sampled_tokens(rng, b, t, z) for _ in range(steps)])
    return {"token_ids": tok, "num_tokens": q, "sampled": sampled}


def config1(seed: int = 1) -> dict:
    """Config 1: B=8, S=2048, V=32000, p=0.5, span U[8,64],
    q ~ U[512, 2048]."""
    return local_config(seed, b=8, s=2048, vocab=32000, p_copy=0.5,
                        span=(8, 64), q_range=(512, 2048))


def config2(seed: int = 2, steps: int = 100, b: int = 256,
            s: int = 8192) -> dict:
    """Config 2: B=256, S=8192, V=128256, p=0.7, span U[16,256],
    q ~ U[2048, 8192], ``steps`` decode steps of 1-5 appended ids."""
    return local_config(seed, b=b, s=s, vocab=128256, p_copy=0.7,
                        span=(16, 256), q_range=(2048, s), steps=steps)


CONFIG2_DRAFTER = dict(k=16, max_pattern_len=32, min_match_len=1,
                       max_occurrences=128, num_backoff=8,
                       max_spec_factor=2.0, max_spec_offset=0.0,
                       min_token_prob=0.1)


def template_docs(rng: np.random.Generator, n_docs: int, doc_len: int,
                  templates: np.ndarray, zipf: Zipf,
                  p_sub: float = 0.05) -> np.ndarray:
    """[n_docs, doc_len] documents: concatenated random templates with a
    ``p_sub`` per-token random substitution."""
    n_t, t_len = templates.shape
    reps = -(-doc_len // t_len)
    pick = rng.integers(0, n_t, size=(n_docs, reps))
    docs = templates[pick].reshape(n_docs, reps * t_len)[:, :doc_len].copy()
    sub = rng.random(docs.shape) < p_sub
    docs[sub] = zipf.draw(rng, int(sub.sum()))
    return docs.astype(np.int32)


def config3(seed: int = 3, n_docs: int = 4096, doc_len: int = 1024,
            n_templates: int = 64, t_len: int = 256, vocab: int = 32000,
            b: int = 64, s: int = 4096, steps: int = 8) -> dict:
    """Config 3: template corpus for the global index plus query rows."""
    rng = np.random.default_rng(seed)
    z = Zipf(1.1, vocab)
    templates = z.draw(rng, (n_templates, t_len))
    corpus_docs = template_docs(rng, n_docs, doc_len, templates, z)
    rows = template_docs(rng, b, s, templates, z)
    q = rng.integers(s // 2, s - 8 * steps, size=b).astype(np.int32)
    sampled = np.stack([sampled_tokens(rng, b, 5, z) for _ in range(steps)])
    return {"corpus_docs": corpus_docs, "token_ids": rows, "num_tokens": q,
            "sampled": sampled}


def config4(seed: int = 4, n: int = 1 << 24, vocab: int = 128256,
            n_queries: int = 1000,
            caps=(32, 16, 8, 4, 2)) -> dict:
    """Config 4: SA build input (50% i.i.d. Zipf(1.1) / 50% copies of
    earlier spans U[32,1024], by token count) plus substring queries."""
    rng = np.random.default_rng(seed)
    z = Zipf(1.1, vocab)
    tokens = copy_stream(rng, n, z, 0.5, 32, 1024, fresh_len=(32, 1024))
    queries = {}
    for c in caps:
        st = rng.integers(0, n - c, size=n_queries)
        queries[c] = tokens[st[:, None] + np.arange(c)[None, :]]
    return {"tokens": tokens, "queries": queries}


CONFIG5_DRAFTER = dict(k=32, max_pattern_len=64, max_occurrences=256,
                       num_backoff=8, enable_global=True,
                       global_capacity=1 << 26, delta_capacity=1 << 16,
                       max_spec_factor=2.0, min_token_prob=0.1)


def config5(seed: int = 5, rank: int = 0, rows: int = 128, s: int = 16384,
            n_docs: int = 65536, doc_len: int = 1023, n_templates: int = 512,
            t_len: int = 512, vocab: int = 128256, steps: int = 32) -> dict:
    """Config 5 (multi-GPU global drafter): a corpus of n_docs template
    documents whose tokens and SEPs fill 2^26 positions, the same on every
    rank (shared seed), and this rank's query rows (rows x s, built the
    same way from new draws) with its decode-step samples."""
    rng = np.random.default_rng(seed)
    z = Zipf(1.1, vocab)
    templates = z.draw(rng, (n_templates, t_len))
    corpus_docs = template_docs(rng, n_docs, doc_len, templates, z)
    rr = np.random.default_rng(seed * 1000 + 17 + rank)
    toks = template_docs(rr, rows, s, templates, z)
    q = rr.integers(s // 2, s - 8 * steps, size=rows).astype(np.int32)
    sampled = np.stack([sampled_tokens(rr, rows, 5, z) for _ in range(steps)])
    return {"corpus_docs": corpus_docs, "token_ids": toks, "num_tokens": q,
            "sampled": sampled}
