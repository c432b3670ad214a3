"""Grammar-constrained greedy sampling on the CPU path, modelled on the reference's sampling
tests (python/lake/engine/tests/test_sampling.py:14-90): greedy takes the largest logit, a token
bitmask restricts it to the allowed ids, and a request with a mask in an overlapped engine is
sampled under its mask while a request without one decodes exactly as in an unconstrained run."""
import torch

from lake_b200.engine.llm_engine import LLMEngine
from lake_b200.ops import core


def _mask(allowed, vocab):
    words = torch.zeros((vocab + 31) // 32, dtype=torch.int64)
    for t in allowed:
        words[t // 32] |= 1 << (t % 32)
    return [int(w) - (1 << 32) if w >= (1 << 31) else int(w) for w in words.tolist()]  # int32 words


def test_greedy_takes_the_largest_logit_and_the_mask_restricts_it():
    logits = torch.tensor([[0.1, 0.9, 0.2, -1.0]])
    assert core.greedy_sample(logits).tolist() == [1]
    bm = torch.tensor([_mask([0, 2], 4)], dtype=torch.int32)
    assert core.greedy_sample(logits, bm).tolist() == [2]
    masked = logits.clone()
    core.apply_token_bitmask(masked, bm)
    assert masked[0, 1] == float("-inf") and masked[0, 3] == float("-inf") and masked[0, 2] == logits[0, 2]


def _engine(**kw):
    return LLMEngine("tiny", device="cpu", max_running=4, max_batched_tokens=128, max_model_len=256, num_blocks=64,
                     **kw)


def test_a_masked_request_obeys_its_mask_and_leaves_the_others_unchanged():
    free_prompt, masked_prompt = list(range(10, 40)), list(range(50, 75))
    want_free = _engine().generate([free_prompt], max_new_tokens=6)[0]
    eng = _engine(overlap=True)
    allowed = [3, 77, 512, 1000]
    a = eng.add_request(free_prompt, max_new_tokens=6)
    b = eng.add_request(masked_prompt, max_new_tokens=6)
    eng.requests[b].bitmask = _mask(allowed, eng.cfg.vocab)
    while eng.has_unfinished():
        eng.step()
    assert eng.requests[a].output == want_free
    assert len(eng.requests[b].output) == 6 and set(eng.requests[b].output) <= set(allowed)
