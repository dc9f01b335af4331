"""Data-parallel request partitioning for one-process-per-GPU serving.

Independent request streams shard across GPUs with no collective on the
per-token path: each rank owns its own engine, KV slot pool and prefix cache,
and only results and statistics travel back over the host.  Two rules decide
where a request runs:

* **prefix affinity** -- requests whose first ``prefix_tokens`` ids agree go to
  the same rank, so the rank that cached the shared prefix reuses it (the
  reference's prefix cache reuses ``min(shared, len - 1)`` positions,
  npu_llm/runtime/generate.py:952-973);
* **balance** -- groups are placed longest-first on the least-loaded rank
  (load = prompt positions + tokens to generate), ties to the lowest rank.
  A prefix group heavier than one rank's fair share is first cut into
  pieces no heavier than that share (members dealt round-robin); each piece
  computes the shared prefix once on its own rank.

The assignment is a pure function of the request list, so every rank computes
the same partition without communicating.
"""

from collections import OrderedDict


def request_load(prompt_ids, new_tokens):
    """Device launches a request costs: one per prompt position, one per
    generated token after the first."""
    return len(prompt_ids) + max(0, new_tokens - 1)


def prefix_key(prompt_ids, prefix_tokens, index):
    """Requests with a full shared prefix (and at least one token after it)
    share a key; every other request gets its own."""
    if prefix_tokens > 0 and len(prompt_ids) > prefix_tokens:
        return ("prefix", tuple(int(t) for t in prompt_ids[:prefix_tokens]))
    return ("single", index)


def assign_ranks(prompts, world, new_tokens, prefix_tokens=16):
    """Rank of every request (list of int, same order as ``prompts``).

    ``new_tokens`` is an int (same for every request) or a list."""
    if world < 1:
        raise ValueError("world must be >= 1")
    n = len(prompts)
    budgets = list(new_tokens) if isinstance(new_tokens, (list, tuple)) else [int(new_tokens)] * n
    if len(budgets) != n:
        raise ValueError("one new_tokens value per request")
    groups = OrderedDict()
    for i, ids in enumerate(prompts):
        groups.setdefault(prefix_key(ids, prefix_tokens, i), []).append(i)
    loads_of = [request_load(prompts[i], budgets[i]) for i in range(n)]
    share = sum(loads_of) / world
    pieces = []
    for members in groups.values():
        load = sum(loads_of[i] for i in members)
        k = max(1, min(len(members), -(-int(load) // max(1, int(share))))) if load > share else 1
        pieces.extend(members[j::k] for j in range(k))
    weighted = []
    for order, members in enumerate(pieces):
        load = sum(loads_of[i] for i in members)
        weighted.append((-load, order, members))
    weighted.sort()
    loads = [0] * world
    ranks = [0] * n
    for neg_load, _, members in weighted:
        target = min(range(world), key=lambda r: (loads[r], r))
        loads[target] += -neg_load
        for i in members:
            ranks[i] = target
    return ranks


def shard(prompts, rank, world, new_tokens, prefix_tokens=16):
    """Indices of the requests this rank serves, in submission order."""
    ranks = assign_ranks(prompts, world, new_tokens, prefix_tokens)
    return [i for i, r in enumerate(ranks) if r == rank]
