"""Draft proposals for speculative decoding (greedy, verified in the next engine step).

Prompt lookup: the last `n` tokens of a request are searched for earlier in its own token
stream (prompt + output); the tokens that followed the most recent earlier match are the
draft. Agentic and retrieval workloads repeat spans of their context, so drafts are often
right; a wrong draft costs only the extra query rows of one step. The engine verifies a
draft by running the request's last token plus the draft as one chunk, sampling every
position, and keeping the longest prefix on which draft and target agree plus one target
token (ops.chain_reject_sample has the same rule for batched device tensors).

Reference parity: the reference schedules `spec` tokens in its SchedulerOutput and has a
chain-reject sampler (python/lake/runtime/scheduler_output.py:82-103,
python/lake/engine/sample/*), but its drafter is an empty placeholder.
"""
from __future__ import annotations


class NgramDrafter:
    """Per-request index of n-gram -> last end position, extended as tokens are appended."""

    def __init__(self, n: int = 3, k: int = 4):
        self.n, self.k = n, k

    def propose(self, req) -> list[int]:
        """Up to k draft tokens following the most recent earlier occurrence of the request's
        last n tokens (empty if none). Reads only the tokens appended since the last call."""
        n, k = self.n, self.k
        L = req.num_tokens
        if L <= n or k <= 0:
            return []
        st = req.meta.get("spec_index")
        if st is None:
            st = req.meta["spec_index"] = {"index": {}, "upto": n - 2}
        index = st["index"]
        # index every n-gram that ends before the current last one (its successor is known)
        first = st["upto"] + 1
        if first < L - 1:
            seg = req.tokens_slice(first - n + 1, L - 1)
            for j in range(len(seg) - n + 1):
                index[tuple(seg[j:j + n])] = first + j
            st["upto"] = L - 2
        hit = index.get(tuple(req.tokens_slice(L - n, L)))
        if hit is None:
            return []
        return req.tokens_slice(hit + 1, min(L, hit + 1 + k))


def accept(draft: list[int], target: list[int]) -> list[int]:
    """Greedy chain rule: target[i] for every position until the first disagreement (the target
    token replaces the draft there), or every draft plus the bonus target token."""
    out = []
    for i, tok in enumerate(draft):
        out.append(target[i])
        if target[i] != tok:
            return out
    out.append(target[len(draft)])
    return out
