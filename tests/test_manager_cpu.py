"""Host logic of the sampling manager and the request parameters (no GPU):
the reference's normalisation (ecahlang/main.py:642-645), the buffer fills of
manager.py:90-97 / :255-268 including bucket padding, and the slot
bookkeeping of manager.py:99-120."""
import numpy as np
import pytest
import torch

from ecahlang_b200.manager import SamplingManager
from ecahlang_b200.parameters import Parameters, normalize
from ecahlang_b200.sampler import repetition_factor

V = 1000


def test_normalize_follows_the_request_layer():
    p = normalize(Parameters(), V)
    assert (p.temperature, p.top_k, p.top_p, p.repetition_penalty) == (1.0, V, 1.0, 1.0)
    p = normalize(Parameters(temperature=0.0, top_k=40, top_p=0.9, repetition_penalty=0.0), V)
    assert p.temperature == 1e-5 and p.top_k == 40 and p.top_p == 0.9 and p.repetition_penalty == 1e-5
    p = normalize(Parameters(frequency_penalty=0.5, presence_penalty=0.25), V)
    assert (p.frequency_penalty, p.presence_penalty) == (0.5, 0.25)


def _mgr():
    m = SamplingManager(V, seq_lens=8, dtype=torch.float16, device="cpu", history_capacity=16, seed=3)
    m.init_sampling_buffers(8)
    return m


def test_fill_sampling_params_writes_rows_and_factors():
    m = _mgr()
    a, b = m.allocate("a"), m.allocate("b")
    m.fill_sampling_params(2, [0.7, 1.0], [50, V], [0.9, 1.0], rep_pens=[1.1, 0.9], batch_ids=["a", "b"])
    assert torch.allclose(m.sampling_temperature_gpu[:2, 0], torch.tensor([0.7, 1.0]))
    assert m.sampling_top_k_gpu[:2].tolist() == [50, V]
    assert np.array_equal(m.sampling_rep_gpu[:2].numpy(), repetition_factor([1.1, 0.9]))
    assert m.sampling_slot_gpu[:2].tolist() == [a, b]
    assert m.sampling_slot_gpu[2:].tolist() == [-1] * 6        # untouched rows keep no slot
    assert not m._fp_eager
    m.fill_sampling_params(1, [1.0], [V], [1.0], freq_pens=[0.5])
    assert m._fp_eager                                      # additive penalties switch on


def test_cuda_graph_fill_resets_padding_rows():
    m = _mgr()
    m.init_cuda_graph_buffers([1, 2, 4])
    m.allocate("x")
    m.fill_cuda_graph_sampling_params(4, 2, [0.5, 0.6], [10, 20], [0.8, 0.7], rep_pens=[1.2, 1.2], batch_ids=["x", "x"])
    m.fill_cuda_graph_sampling_params(4, 1, [0.9], [5], [0.5])
    assert torch.allclose(m._cg_temperature[4][:, 0], torch.tensor([0.9, 1.0, 1.0, 1.0]))
    assert m._cg_top_k[4].tolist() == [5, V, V, V]
    assert m._cg_top_p[4].tolist() == [0.5, 1.0, 1.0, 1.0]
    assert m._cg_rep[4].tolist() == [1.0] * 4
    assert m._cg_slot[4].tolist() == [-1] * 4


def test_slots_are_recycled_and_reset():
    m = _mgr()
    s = m.allocate("r1")
    m.penalty.load(s, [3, 4], [1, 2])
    assert int(m.penalty.slot_len[s]) == 2
    m.free("r1")
    s2 = m.allocate("r2")
    assert s2 == s and int(m.penalty.slot_len[s2]) == 0     # the reused slot starts empty
    m.free("missing")                                      # freeing an unknown id is a no-op
    assert m.seq_lens == 128                               # at least 128 slots, as manager.py:31
    for i in range(len(m.free_seq_lens)):
        m.allocate(f"q{i}")
    with pytest.raises(RuntimeError):
        m.allocate("one-too-many")


def test_sample_has_no_cpu_path():
    m = _mgr()
    m.fill_sampling_params(2, [1.0, 1.0], [V, V], [1.0, 1.0])
    with pytest.raises(RuntimeError, match="CUDA"):
        m.sample(torch.zeros(2, V, dtype=torch.float16))


def test_bucket_captured_without_additive_penalties_refuses_them():
    """A CUDA graph replays the launch it captured: a bucket captured with the
    frequency/presence penalties off must refuse them later, loudly."""
    m = _mgr()
    m.init_cuda_graph_buffers([2, 4])
    m._cg_captured_fp[2] = False          # what sample() records while capturing
    m.fill_cuda_graph_sampling_params(2, 1, [1.0], [V], [1.0])            # none requested: fine
    with pytest.raises(RuntimeError, match="captured"):
        m.fill_cuda_graph_sampling_params(2, 1, [1.0], [V], [1.0], freq_pens=[0.5])
    m.fill_cuda_graph_sampling_params(4, 1, [1.0], [V], [1.0], freq_pens=[0.5])   # never captured
    m2 = SamplingManager(V, seq_lens=8, dtype=torch.float16, device="cpu", history_capacity=16,
                         freq_pres_in_graphs=True)
    m2.init_sampling_buffers(8)
    m2.init_cuda_graph_buffers([2])
    m2._cg_captured_fp[2] = True
    m2.fill_cuda_graph_sampling_params(2, 1, [1.0], [V], [1.0], pres_pens=[0.3])


def test_full_penalty_history_is_reported():
    """A slot whose history filled up (overflow flag copied back after the
    update) makes the next fill for that request raise."""
    m = _mgr()
    s = m.allocate("r")
    m.fill_sampling_params(1, [1.0], [V], [1.0], rep_pens=[1.1], batch_ids=["r"])
    m._overflow_host[s] = 1               # what update_penalties copies back
    with pytest.raises(RuntimeError, match="full"):
        m.fill_sampling_params(1, [1.0], [V], [1.0], rep_pens=[1.1], batch_ids=["r"])
    m.free("r")
    s2 = m.allocate("r2")
    assert s2 == s
    m.fill_sampling_params(1, [1.0], [V], [1.0], rep_pens=[1.1], batch_ids=["r2"])   # reset on allocate
