"""The vLLM glue (suffixgpu_b200/vllm_adapter.py): config mapping and the
class contract on CPU; on the GPU, the adapter's propose through vLLM's
ngram_gpu call sequence equals the oracle drafter, and install() harvests
finished requests into the global index."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

vllm_adapter = pytest.importorskip("suffixgpu_b200.vllm_adapter")


def _config(k=4, lookup_max=8, lookup_min=1, factor=1.0, min_prob=0.1,
            cached=10000, max_model_len=256, max_num_seqs=8):
    spec = SimpleNamespace(num_speculative_tokens=k,
                           prompt_lookup_max=lookup_max,
                           prompt_lookup_min=lookup_min,
                           suffix_decoding_max_spec_factor=factor,
                           suffix_decoding_min_token_prob=min_prob,
                           suffix_decoding_max_cached_requests=cached)
    return SimpleNamespace(
        speculative_config=spec,
        model_config=SimpleNamespace(max_model_len=max_model_len),
        scheduler_config=SimpleNamespace(max_num_seqs=max_num_seqs))


def test_config_mapping_reads_vllm_fields():
    from vllm.config import SpeculativeConfig
    fields = SpeculativeConfig.__dataclass_fields__
    for name in ("num_speculative_tokens", "prompt_lookup_max",
                 "prompt_lookup_min", "suffix_decoding_max_spec_factor",
                 "suffix_decoding_min_token_prob",
                 "suffix_decoding_max_cached_requests"):
        assert name in fields
    kw = vllm_adapter.drafter_kwargs(_config(k=5, lookup_max=24,
                                             lookup_min=2, factor=2.0,
                                             min_prob=0.25))
    assert (kw["k"], kw["max_pattern_len"], kw["min_match_len"]) == (5, 24, 2)
    assert (kw["max_spec_factor"], kw["min_token_prob"]) == (2.0, 0.25)
    assert kw["enable_global"] is True
    kw = vllm_adapter.drafter_kwargs(_config(cached=0, lookup_max=None),
                                     max_occurrences=64)
    assert kw["enable_global"] is False and kw["max_pattern_len"] == 32
    assert kw["max_occurrences"] == 64


def test_proposer_is_an_ngram_gpu_proposer():
    from vllm.v1.spec_decode.ngram_proposer_gpu import NgramProposerGPU
    assert issubclass(vllm_adapter.SuffixGPUProposer, NgramProposerGPU)
    # the runner's ngram_gpu branch calls these two; both are ours
    for name in ("update_token_ids_ngram", "propose"):
        assert getattr(vllm_adapter.SuffixGPUProposer, name) is not \
            getattr(NgramProposerGPU, name)


@pytest.mark.gpu
def test_prepare_matches_vllm_update_token_ids_ngram():
    """The one-launch update_token_ids_ngram equals vLLM's own torch-op
    version on the same inputs: discarded rows, -1 inside a row (not
    left-aligned), ids at or above the vocabulary size, empty counts whose
    next id falls back to the last committed token (count 0 too), a
    sliced persistent batch; the ragged list form goes to vLLM's code."""
    from vllm.v1.spec_decode.ngram_proposer_gpu import NgramProposerGPU
    dev = torch.device("cuda")
    prop = vllm_adapter.SuffixGPUProposer(_config(cached=0), dev)
    rng = np.random.default_rng(8)
    for trial in range(6):
        max_reqs, s = 40, 300
        b = int(rng.integers(1, max_reqs + 1))
        t = int(rng.integers(1, 7))
        vocab = 50
        tok = torch.from_numpy(rng.integers(
            0, vocab, size=(max_reqs, s)).astype(np.int32)).to(dev)
        n = torch.from_numpy(rng.integers(
            0, s + 1, size=max_reqs).astype(np.int32)).to(dev)
        samp = rng.integers(0, vocab + 5, size=(b, t)).astype(np.int32)
        samp[rng.random((b, t)) < 0.35] = -1
        if trial % 2:  # left-aligned accepted tokens, as the sampler emits
            for r in range(b):
                bad = np.nonzero(samp[r] == -1)[0]
                if bad.size:
                    samp[r, bad[0]:] = -1
        samp_d = torch.from_numpy(samp).to(dev)
        disc = torch.from_numpy(rng.random(max_reqs) < 0.2).to(dev)
        batch = SimpleNamespace(num_reqs=b, vocab_size=vocab)
        got = prop.update_token_ids_ngram(samp_d, batch, tok, n, disc)
        exp = NgramProposerGPU.update_token_ids_ngram(prop, samp_d, batch,
                                                      tok, n, disc)
        for g, e in zip(got, exp):
            assert g.dtype == e.dtype and g.shape == e.shape
            torch.testing.assert_close(g, e, rtol=0, atol=0)
    ragged = [[1, 2], [], [3]]
    batch = SimpleNamespace(num_reqs=3, vocab_size=50)
    got = prop.update_token_ids_ngram(ragged, batch, tok, n, disc)
    exp = NgramProposerGPU.update_token_ids_ngram(prop, ragged, batch, tok,
                                                  n, disc)
    for g, e in zip(got, exp):
        torch.testing.assert_close(g, e, rtol=0, atol=0)


@pytest.mark.gpu
def test_propose_matches_oracle_through_vllm_sequence():
    """Four decode steps through update_token_ids_ngram + propose, as the
    runner's ngram_gpu branch calls them, against the oracle drafter fed
    the same sampled ids."""
    from oracle import suffix_oracle as so
    dev = torch.device("cuda")
    rng = np.random.default_rng(5)
    b, s, k = 6, 256, 4
    cfg = _config(k=k, lookup_max=8, factor=1.0, min_prob=0.1,
                  max_model_len=200)
    prop = vllm_adapter.SuffixGPUProposer(cfg, dev)
    kw = vllm_adapter.drafter_kwargs(cfg)
    ref = so.SuffixDrafter(**{x: kw[x] for x in (
        "k", "max_pattern_len", "min_match_len", "max_occurrences",
        "enable_global", "global_capacity", "delta_capacity",
        "max_spec_factor", "min_token_prob", "num_backoff")})
    base = rng.integers(0, 5, size=(b, s)).astype(np.int32)
    base[:, 40:80] = base[:, 0:40]  # repeats to match
    n_host = np.array([100, 150, 1, 0, 199, 120], dtype=np.int32)
    tok_g = torch.from_numpy(base.copy()).to(dev)
    tok_o = base.copy()
    n_g = torch.from_numpy(n_host.copy()).to(dev)
    n_o = n_host.copy()
    batch = SimpleNamespace(num_reqs=b, vocab_size=5)
    discard = torch.zeros(b, dtype=torch.bool, device=dev)
    for step in range(4):
        sampled = rng.integers(0, 5, size=(b, k + 1)).astype(np.int32)
        sampled[rng.random((b, k + 1)) < 0.3] = -1
        # accepted tokens are left-aligned: -1 after the first -1
        for r in range(b):
            bad = np.nonzero(sampled[r] == -1)[0]
            if bad.size:
                sampled[r, bad[0]:] = -1
        sampled_g = torch.from_numpy(sampled).to(dev)
        _, counts, valid = prop.update_token_ids_ngram(
            sampled_g, batch, tok_g, n_g, discard)
        draft, nv = prop.propose(n_g, tok_g, valid, counts)
        cnt = (sampled != -1).sum(axis=1)
        d_o, nv_o, new_o = ref.propose_with_update(n_o, tok_o, sampled, cnt,
                                                   max_model_len=200)
        np.testing.assert_array_equal(draft.cpu().numpy(), d_o)
        np.testing.assert_array_equal(nv.cpu().numpy(), nv_o)
        np.testing.assert_array_equal(tok_g.cpu().numpy(), tok_o)
        # the runner advances its counts from the valid counts
        n_g = (n_g + counts).to(torch.int32)
        n_o = new_o


@pytest.mark.gpu
def test_install_harvests_finished_requests():
    """install() replaces the runner's drafter and harvests the rows of
    finished requests (host lengths) before the runner's own update."""
    from oracle import suffix_oracle as so
    dev = torch.device("cuda")
    rng = np.random.default_rng(6)
    rows = rng.integers(0, 9, size=(4, 64)).astype(np.int32)
    calls = []
    runner = SimpleNamespace(
        vllm_config=_config(k=3, lookup_max=8, max_model_len=64),
        device=dev, drafter=None,
        token_ids_gpu_tensor=torch.from_numpy(rows).to(dev),
        input_batch=SimpleNamespace(
            req_id_to_index={"a": 0, "b": 1, "c": 2, "d": 3},
            num_tokens_no_spec=np.array([10, 20, 0, 33], dtype=np.int32)),
        _update_states=lambda so_: calls.append(so_))
    prop = vllm_adapter.install(runner, rebuild_threshold=1 << 20)
    assert runner.drafter is prop
    out = SimpleNamespace(finished_req_ids={"b", "d", "zz"})
    runner._update_states(out)
    assert calls == [out]
    gi = prop.drafter.global_index
    o = so.GlobalIndex(capacity=1 << 22, delta_capacity=1 << 16, k=3,
                       max_occurrences=128, rebuild_threshold=1 << 20)
    harvested = sorted(["b", "d"], key=lambda r: list(
        out.finished_req_ids).index(r))
    idx = {"b": 1, "d": 3}
    n = {"b": 20, "d": 33}
    o.append_documents([rows[idx[r], :n[r]] for r in harvested])
    assert gi.delta_len == o.delta_len == 20 + 33 + 2
    np.testing.assert_array_equal(gi.delta[:gi.delta_len].cpu().numpy(),
                                  o.delta[:o.delta_len])
