"""Host-side pieces: SamplingParams validation (the reference's own checks,
``tests/test_host.py:47-50`` of QEdge, plus the new fields), the per-row
packing of SamplingBatch and the ModelRunner installation shim."""
from types import SimpleNamespace

import pytest
import torch

from qedge_b200.batch import SamplingBatch
from qedge_b200.sampling_params import SamplingParams


@pytest.mark.parametrize("kwargs", [{"top_p": 0}, {"top_p": 1.1}, {"min_p": -0.1},
                                    {"min_tokens": 3, "max_tokens": 2}, {"temperature": -1},
                                    {"top_k": 0}, {"repetition_penalty": 0.0}, {"seed": -1}])
def test_sampling_params_reject_invalid(kwargs):
    with pytest.raises(ValueError):
        SamplingParams(**kwargs)


def test_sampling_params_defaults_match_reference():
    p = SamplingParams()
    assert (p.temperature, p.top_p, p.top_k, p.min_p, p.max_tokens, p.min_tokens, p.ignore_eos) == \
        (0.0, None, None, None, 128, 0, False)
    assert p.repetition_penalty == 1.0 and p.seed is None


def seq(t, p=None, k=None, rp=1.0, ids=()):
    return SimpleNamespace(temperature=t, top_p=p, top_k=k, min_p=None, repetition_penalty=rp,
                           token_ids=list(ids))


def test_batch_packing_and_flags():
    b = SamplingBatch(max_bs=4, vocab_size=100, device="cpu", history_width=3)
    b.fill([seq(0.0), seq(0.7, 0.9, 5), seq(1.0, None, -1, 1.2, [1, 2, 3, 4])])
    assert b.temperatures[:3].tolist() == pytest.approx([0.0, 0.7, 1.0])
    assert b.top_ps[:3].tolist() == pytest.approx([1.0, 0.9, 1.0])
    assert b.top_ks[:3].tolist() == [100, 5, 100]          # None / <=0 -> vocab (batch.py:154-157)
    assert b.rep_penalties[:3].tolist() == pytest.approx([1.0, 1.0, 1.2])
    assert not b.all_greedy and b.any_greedy and b.use_top_k and b.use_top_p and b.use_penalty
    assert b.history_lens[:3].tolist() == [0, 0, 3]
    assert b.history[2].tolist() == [2, 3, 4]               # last `history_width` ids
    kw = b.sampler_kwargs(3)
    assert set(kw) == {"top_ks", "rep_penalties", "history", "history_lens"}


def test_batch_signature_cache_skips_upload():
    b = SamplingBatch(max_bs=2, vocab_size=10, device="cpu")
    seqs = [seq(0.5, 0.8)]
    b.fill(seqs)
    b.temperatures.fill_(9.0)       # a second fill with the same params must not re-upload
    b.fill(seqs)
    assert b.temperatures[0].item() == 9.0
    with pytest.raises(ValueError):
        b.fill([seq(1.0)] * 3)


def test_install_shim_wires_runner(monkeypatch):
    from qedge_b200 import integration, sampler as S

    class FakeSampler:
        def __init__(self, seed=0):
            self.calls = []

        def __call__(self, logits, t, p, **kw):
            self.calls.append((logits.shape, kw))
            return torch.zeros(logits.shape[0], dtype=torch.long)

    monkeypatch.setattr(integration, "QESampler", FakeSampler)
    runner = SimpleNamespace(batch=SimpleNamespace(max_bs=300, vocab_size=50), device="cpu",
                             sampler="orig", _sample_gpu="orig_fn",
                             sample_cpu=torch.empty(256, dtype=torch.int64))
    integration.install(runner, seed=3, history_width=4)
    assert runner.sample_cpu.numel() == 300
    ids = runner._sample_gpu([torch.zeros(2, 50)], [seq(0.0), seq(1.0, 0.5, None, 1.1, [7])])
    assert ids.tolist() == [0, 0] and runner.qe_step == 1
    shape, kw = runner.sampler.calls[0]
    assert shape == (2, 50) and kw["use_top_p"] and kw["step"] == 0 and "history" in kw
    integration.uninstall(runner)
    assert runner.sampler == "orig" and runner._sample_gpu == "orig_fn"


def test_batch_packs_per_request_seeds_and_min_p():
    b = SamplingBatch(max_bs=3, vocab_size=100, device="cpu")
    b.default_seed = 7
    s0 = seq(1.0)
    s1 = seq(0.8, 0.9)
    s1.seed = 2**64 - 1
    s1.min_p = 0.05
    b.fill([s0, s1])
    kw = b.sampler_kwargs(2)
    assert "seeds" in kw and "min_ps" in kw
    assert kw["seeds"].tolist() == [7, -1]              # uint64 bit patterns in int64
    assert abs(kw["min_ps"][1].item() - 0.05) < 1e-7
