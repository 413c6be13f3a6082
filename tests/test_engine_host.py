"""Engine layer on the host: GPT initialisation and scheduler semantics (no GPU).

The GPT weights drawn by ``torch.manual_seed(s); GptModel(cfg)`` must equal the
reference's (the sha256 digests of its state_dict recorded in
tests/golden/engine_golden.pt), so the greedy-token comparison on the GPU runs
the reference's model.  Scheduler cases follow the behaviour of the
reference's scheduler.py:30-57 and 139-176.
"""

import hashlib

import pytest
import torch

from nifre_b200.data_model import InferenceRequest, RequestState
from nifre_b200.gpt import GptModel
from nifre_b200.scheduler import Scheduler


def _digest(model):
    return {n: (tuple(p.shape), hashlib.sha256(p.detach().contiguous().numpy().tobytes()).hexdigest())
            for n, p in model.state_dict().items()}


@pytest.mark.parametrize("name", ["tiny", "gpt124m_cfg1"])
def test_gpt_init_matches_reference_weights(golden_engine, name):
    case = golden_engine[name]
    torch.manual_seed(case["seed"])
    model = GptModel(case["cfg"])
    assert _digest(model) == case["digest"]


def _req(rid, n_prompt, max_new=4, chunk=4):
    return InferenceRequest(request_id=rid, prompt_token_ids=list(range(n_prompt)), max_new_tokens=max_new,
                            prefill_chunk_size=chunk)


def test_scheduler_slots_fifo_and_budget():
    s = Scheduler(max_concurrent_requests=2, max_tokens_per_step=6)
    a, b, c = _req("a", 10), _req("b", 3), _req("c", 5)
    for r in (a, b, c):
        s.add_request(r)
    res = s.schedule()
    # a's chunk (4) fits the budget of 6; b's (3) then does not and is skipped
    assert [r.request_id for r in res.prefill_requests] == ["a"]
    assert a.batch_idx == 0 and b.batch_idx == 1 and c.state is RequestState.WAITING


def test_scheduler_decode_first_and_skip_not_stop():
    s = Scheduler(max_concurrent_requests=3, max_tokens_per_step=5)
    a, b, c = _req("a", 8), _req("b", 2), _req("c", 8)
    for r in (a, b, c):
        s.add_request(r)
    s.schedule()
    # a decodes; b still prefilling with 2 left; c has 8 left (chunk 4)
    a.prefill_offset = 8
    s.mark_prefill_done(a)
    b.prefill_offset = 0
    res = s.schedule()
    assert [r.request_id for r in res.decode_requests] == ["a"]
    # budget 5 - 1 = 4: b's chunk (2) fits, c's chunk (4) no longer fits after b -> skipped
    assert [r.request_id for r in res.prefill_requests] == ["b"]


def test_scheduler_finish_returns_slot_to_end():
    s = Scheduler(max_concurrent_requests=3)
    reqs = [_req(str(i), 1, max_new=1) for i in range(3)]
    for r in reqs:
        s.add_request(r)
    s.schedule()
    r0 = reqs[0]
    r0.prefill_offset = 1
    s.mark_prefill_done(r0)
    s.mark_decode_done(r0, 7)
    assert r0.state is RequestState.FINISHED and r0.output_token_ids == [7]
    assert s.free_slots == [0] and r0.batch_idx is None
    s.add_request(_req("x", 2))
    s.schedule()
    assert s.running["x"].batch_idx == 0


def test_scheduler_cancel_and_errors():
    s = Scheduler(max_concurrent_requests=1)
    a, b = _req("a", 3), _req("b", 3)
    s.add_request(a)
    s.add_request(b)
    s.schedule()
    assert s.cancel_request("b").status == "timeout" and "b" in s.failed
    assert s.cancel_request("a").batch_idx is None and s.free_slots == [0]
    with pytest.raises(KeyError):
        s.cancel_request("zz")
    with pytest.raises(ValueError):
        Scheduler(0)
    with pytest.raises(ValueError):
        s.mark_decode_done(_req("q", 1), 1)
