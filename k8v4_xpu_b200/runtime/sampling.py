"""Random sampling of next tokens (temperature, top-k, top-p, seed).

The reference serves through stock vLLM, whose requests may sample instead
of taking the argmax. Greedy rows stay on the argmax kernel inside the
captured decode graphs; a step with at least one sampling row runs eagerly
and draws those rows here from the full-vocabulary logits (under tensor
parallelism every rank gathers the vocabulary shards, then draws with the
same per-sequence generator, so the ranks agree).

Each sequence owns a ``torch.Generator`` on the device, seeded with the
request's ``seed``; without one the seed is derived from the engine seed
and the sequence id, which every rank of a TP or CP group shares.
"""
from __future__ import annotations

import torch

_MIX = 0x9E3779B97F4A7C15  # odd 64-bit constant (golden ratio) to spread seq ids


def samples(params) -> bool:
    """Whether a request samples (temperature above zero) instead of taking the argmax."""
    return params is not None and (params.temperature or 0.0) > 0.0


def seed_for(params, engine_seed: int, seq_id: int) -> int:
    if params.seed is not None:
        return int(params.seed) & ((1 << 63) - 1)
    return ((int(engine_seed) + 1) * _MIX + int(seq_id) * 0x2545F4914F6CDD1D) & ((1 << 63) - 1)


def generator_for(seq, engine_seed: int, device) -> torch.Generator:
    """The sequence's generator, created and seeded on first use."""
    g = getattr(seq, "generator", None)
    if g is None:
        g = torch.Generator(device=device)
        g.manual_seed(seed_for(seq.params, engine_seed, seq.seq_id))
        seq.generator = g
    return g


def filter_logits(x: torch.Tensor, top_k: int, top_p: float, min_p: float = 0.0) -> torch.Tensor:
    """One row of fp32 logits (already divided by the temperature) with the
    tokens outside the top-k, outside the top-p nucleus, and below ``min_p``
    times the most likely token's probability set to -inf. The most likely
    token always stays."""
    V = x.shape[-1]
    if 0.0 < min_p <= 1.0:
        p = torch.softmax(x, -1)
        x = torch.where(p < min_p * p.max(), torch.full_like(x, float("-inf")), x)
    if 0 < top_k < V:
        kth = torch.topk(x, top_k).values[-1]
        x = torch.where(x < kth, torch.full_like(x, float("-inf")), x)
    if 0.0 < top_p < 1.0:
        vals, idx = torch.sort(x, descending=True)
        p = torch.softmax(vals, -1)
        before = torch.cumsum(p, -1) - p          # mass of the tokens ranked above each one
        drop = before >= top_p
        drop[0] = False
        x = x.clone()
        x[idx[drop]] = float("-inf")
    return x


def sample_rows(logits: torch.Tensor, params: list, gens: list) -> torch.Tensor:
    """Token ids [R] (int64) for logits [R, V]: rows whose params sample are
    drawn from softmax(filtered logits / temperature) with their generator;
    the others take the argmax."""
    lg = logits.float()
    out = torch.argmax(lg, dim=-1)
    for i, (p, g) in enumerate(zip(params, gens)):
        if not samples(p):
            continue
        probs = torch.softmax(_filtered(lg[i], p), -1)
        out[i] = torch.multinomial(probs, 1, generator=g)[0]
    return out


def probs_rows(logits: torch.Tensor, p) -> torch.Tensor:
    """Sampling distribution [R, V] (fp32) of the rows of ``logits`` under one
    request's temperature, top-k and top-p."""
    lg = logits.float()
    return torch.stack([torch.softmax(_filtered(lg[j], p), -1) for j in range(lg.shape[0])])


def _filtered(row: torch.Tensor, p) -> torch.Tensor:
    return filter_logits(row / float(p.temperature), int(p.top_k or 0), float(p.top_p if p.top_p else 1.0),
                         float(getattr(p, "min_p", 0.0) or 0.0))


def speculative_sample(logits: torch.Tensor, drafts: torch.Tensor, p, gen: torch.Generator) -> tuple[int, int]:
    """Speculative sampling of one sequence's verify rows.

    ``logits`` [k + 1, V]: row j scores the token after verify row j (row 0
    is the last committed token, rows 1..k the drafts); ``drafts`` [k]. The
    drafter proposes deterministically (its argmax: all its mass on one
    token), so draft j is kept with probability p_j(draft j) under the
    target's sampling distribution p_j, and the first rejected position draws
    from p_j with the rejected token removed (renormalized); after k kept
    drafts the bonus token draws from p_k. The emitted tokens then have the
    target's sampling distribution at every position (the standard
    speculative sampling argument with a one-point draft distribution).
    Returns (accepted drafts a, the token drawn at position a)."""
    k = drafts.shape[0]
    probs = probs_rows(logits, p)
    u = torch.rand(k, generator=gen, device=gen.device) if k else None
    a = 0
    while a < k and float(u[a]) < float(probs[a, drafts[a]]):
        a += 1
    if a < k:
        res = probs[a].clone()
        res[drafts[a]] = 0.0
        if float(res.sum()) <= 0.0:  # the target puts all its mass on the rejected token (u hit the edge)
            res = probs[a]
        x = torch.multinomial(res / res.sum(), 1, generator=gen)[0]
    else:
        x = torch.multinomial(probs[k], 1, generator=gen)[0]
    return a, int(x)


def wants_logprobs(params) -> bool:
    """Whether a request asks for the log-probabilities of its tokens."""
    return params is not None and getattr(params, "logprobs", None) is not None


def needs_logits(params) -> bool:
    """Requests whose steps need the full-vocabulary logits (so they run
    eagerly): sampling ones, the ones asking for log-probabilities and the
    ones with logits processors. Asked every decode step for every sequence,
    so the answer is kept on the (unchanging) params object."""
    if params is None:
        return False
    memo = params.__dict__.get("_needs_logits")
    if memo is None:
        memo = samples(params) or wants_logprobs(params) or has_processors(params)
        params.__dict__["_needs_logits"] = memo
    return memo


def logprob_entry(row_logits: torch.Tensor, token: int, top_n: int) -> tuple:
    """(log-probability of ``token``, [(id, log-probability)] of the ``top_n``
    most likely tokens) under the model's distribution (the raw logits, before
    temperature and filtering, as vLLM reports them)."""
    lsm = torch.log_softmax(row_logits.float(), -1)
    top = []
    if top_n:
        v, i = torch.topk(lsm, int(top_n))
        top = list(zip(i.tolist(), v.tolist()))
    return float(lsm[int(token)]), top


def stash_of(engine) -> dict:
    """Per-sequence log-probability entries waiting for the commit of their tokens."""
    return engine.__dict__.setdefault("_lp_next", {})


def record(engine, seq) -> None:
    """Append the next waiting entry (or None) to a sequence that asked for
    log-probabilities, for the token just appended to its output."""
    if wants_logprobs(seq.params):
        stash = stash_of(engine)
        lst = stash.get(seq.seq_id)
        seq.logprobs.append(lst.pop(0) if lst else None)
        if not lst:
            stash.pop(seq.seq_id, None)


def wants_prompt_logprobs(params) -> bool:
    """Whether a request asks for the log-probabilities of its prompt tokens."""
    return params is not None and getattr(params, "prompt_logprobs", None) is not None


def logprob_rows(logits: torch.Tensor, tokens: list[int], top_n: int) -> list[tuple]:
    """:func:`logprob_entry` of many rows at once: row i scores ``tokens[i]``."""
    lsm = torch.log_softmax(logits.float(), -1)
    idx = torch.tensor(tokens, dtype=torch.int64, device=lsm.device).view(-1, 1)
    lp = lsm.gather(1, idx).view(-1).tolist()
    if top_n:
        v, i = torch.topk(lsm, int(top_n), dim=-1)
        tops = [list(zip(a, b)) for a, b in zip(i.tolist(), v.tolist())]
    else:
        tops = [[] for _ in tokens]
    return list(zip(lp, tops))


def has_processors(params) -> bool:
    """Whether a request changes its logits before the choice: repetition /
    presence / frequency penalties, a logit bias, or a minimum length that
    holds back its stop tokens."""
    return params is not None and (float(getattr(params, "repetition_penalty", 1.0)) != 1.0
                                   or float(getattr(params, "presence_penalty", 0.0)) != 0.0
                                   or float(getattr(params, "frequency_penalty", 0.0)) != 0.0
                                   or bool(getattr(params, "logit_bias", None))
                                   or int(getattr(params, "min_tokens", 0) or 0) > 0
                                   or bool(getattr(params, "allowed_sequences", None)))


def _prompt_mask(prompt, V: int, dev, holder=None) -> torch.Tensor:
    """Tokens of the prompt as a [V] bool mask, kept on ``holder`` (the
    sequence) so that a long prompt is turned into a mask once."""
    key = (V, str(dev))
    cached = getattr(holder, "_prompt_mask", None) if holder is not None else None
    if cached is not None and cached[0] == key:
        return cached[1]
    seen = torch.zeros(V, dtype=torch.bool, device=dev)
    if len(prompt):
        seen[torch.tensor(list(prompt), dtype=torch.int64, device=dev)] = True
    if holder is not None:
        holder._prompt_mask = (key, seen)
    return seen


def process_row(row: torch.Tensor, prompt, output: list[int], p, holder=None) -> torch.Tensor:
    """Processed fp32 logits of one row, as vLLM defines the processors:
    ``repetition_penalty`` r divides a positive logit (multiplies a negative
    one) of every token seen in the prompt or the output; ``presence_penalty``
    subtracts a constant from tokens the output holds, ``frequency_penalty``
    that constant times how often the output holds them; ``logit_bias`` adds
    its value to its token; while the output is shorter than ``min_tokens``
    the stop tokens are held back (-inf). ``holder`` (the sequence) keeps the
    prompt's token mask between steps."""
    x = row.float().clone()
    V = x.shape[-1]
    dev = x.device
    out = torch.tensor(output, dtype=torch.int64, device=dev) if output else None
    r = float(getattr(p, "repetition_penalty", 1.0))
    if r != 1.0:
        seen = _prompt_mask(prompt, V, dev, holder).clone()
        if out is not None:
            seen[out] = True
        x = torch.where(seen, torch.where(x > 0, x / r, x * r), x)
    if out is not None:
        counts = torch.bincount(out, minlength=V)[:V].to(x.dtype)
        x = x - float(getattr(p, "frequency_penalty", 0.0)) * counts \
            - float(getattr(p, "presence_penalty", 0.0)) * (counts > 0).to(x.dtype)
    bias = [(int(t), float(v)) for t, v in (getattr(p, "logit_bias", None) or {}).items() if 0 <= int(t) < V]
    if bias:
        ids = torch.tensor([t for t, _ in bias], dtype=torch.int64, device=dev)
        x[ids] += torch.tensor([v for _, v in bias], dtype=x.dtype, device=dev)
    if len(output) < int(getattr(p, "min_tokens", 0) or 0) and p.stop_token_ids:
        stops = [int(t) for t in p.stop_token_ids if 0 <= int(t) < V]
        if stops:
            x[torch.tensor(stops, dtype=torch.int64, device=dev)] = float("-inf")
    allowed = choice_continuations(p, output)
    if allowed is not None:
        ids = [t for t in allowed if 0 <= t < V]
        if ids:
            keep = torch.full_like(x, float("-inf"))
            idx = torch.tensor(ids, dtype=torch.int64, device=dev)
            keep[idx] = x[idx]
            x = keep
    return x


def choice_continuations(p, output) -> set | None:
    """Guided choice: the tokens that keep ``output`` a prefix of one of the
    allowed sequences (plus the stop tokens when it already equals one), or
    None when the request is not guided."""
    seqs = getattr(p, "allowed_sequences", None)
    if not seqs:
        return None
    n = len(output)
    out = list(output)
    nxt, complete = set(), False
    for s in seqs:
        if list(s[:n]) == out:
            if len(s) > n:
                nxt.add(int(s[n]))
            else:
                complete = True
    if complete:
        nxt |= {int(t) for t in (p.stop_token_ids or ())}
    return nxt


def choice_finished(p, output) -> bool:
    """Guided choice: the output equals an allowed sequence that no other one extends."""
    seqs = getattr(p, "allowed_sequences", None)
    if not seqs:
        return False
    out = list(output)
    return any(list(s) == out for s in seqs) and not any(len(s) > len(out) and list(s[:len(out)]) == out
                                                         for s in seqs)
