"""OpenAI-compatible HTTP server (FastAPI).

Endpoints: ``POST /v1/chat/completions`` and ``POST /v1/completions``
(streaming as server-sent events, ``stream_options.include_usage`` and
``continuous_usage_stats``), ``GET /v1/models``, ``GET /health`` (``/ping``), ``GET /version``,
``POST /tokenize``, ``POST /detokenize`` and
``GET /metrics`` (Prometheus, ``vllm:*`` names). This is the surface the
reference's clients use against stock vLLM (``bench/serve_coding.py:27-45``,
``launch.sh:219-232``). A request without ``temperature`` (or with 0)
decodes greedily, the benchmark path of the reference; ``temperature`` > 0
samples, with ``top_p``, ``top_k`` (0 or -1: off), ``min_p`` and ``seed``;
the repetition, presence and frequency penalties, ``logit_bias`` and
``min_tokens`` apply to either
(``runtime.sampling``; under MTP the drafts are verified by speculative
sampling). Stop
strings (``stop``) end a request before the first match, in streamed and
whole responses, and drop its sequence from the engine. ``logprobs``
(completions: the top-N count; chat: ``logprobs`` + ``top_logprobs``) gives
each token's log-probability under the model's logits; with ``echo`` the
prompt comes back first, with its tokens' log-probabilities when asked
(computed during the prefill, which then takes no prefix-cache hit). ``n`` (1-16)
choices run as n engine requests over the same prompt (seed + i for choice
i of a seeded request); ``best_of`` runs that many and returns the n with
the highest cumulative log-probability. ``guided_choice`` confines the
output to one of the given strings (as the tokenizer encodes them). Beam
search, structured output (``response_format``, JSON / regex guided
decoding) and tool calls are not built: such
requests get a 400 instead of being served as if the field were absent.
"""
from __future__ import annotations

import asyncio
import dataclasses
import json
import time
import uuid
from typing import Any

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, Response, StreamingResponse
from prometheus_client import CONTENT_TYPE_LATEST
from pydantic import BaseModel, Field

from ..runtime.scheduler import SamplingParams
from .tokenizer import IncrementalDecoder, StopMatcher


class StreamOptions(BaseModel):
    include_usage: bool = False
    continuous_usage_stats: bool = False


class _Common(BaseModel):
    model: str | None = None
    max_tokens: int | None = None
    max_completion_tokens: int | None = None
    stream: bool = False
    stream_options: StreamOptions | None = None
    ignore_eos: bool = False
    stop_token_ids: list[int] = Field(default_factory=list)
    stop: str | list[str] | None = None
    include_stop_str_in_output: bool = False
    logprobs: int | bool | None = None   # completions: top-N count; chat: on / off
    top_logprobs: int | None = None      # chat: top-N count
    temperature: float | None = None
    top_p: float | None = None
    top_k: int | None = None
    seed: int | None = None
    min_p: float | None = None
    logit_bias: dict[str, float] | None = None
    min_tokens: int | None = None
    repetition_penalty: float | None = None
    presence_penalty: float | None = None
    frequency_penalty: float | None = None
    n: int = 1
    # accepted only in their neutral form: refused with a 400 rather than ignored
    best_of: int | None = None
    use_beam_search: bool = False
    response_format: dict | None = None
    tools: list | None = None
    guided_json: Any = None
    guided_regex: str | None = None
    guided_choice: list | None = None


class CompletionRequest(_Common):
    prompt: str | list[int] | list[str]
    echo: bool = False  # the prompt comes back before the completion (with its logprobs when asked)


class ChatMessage(BaseModel):
    role: str
    content: Any = ""


class ChatRequest(_Common):
    messages: list[ChatMessage]


class TokenizeRequest(BaseModel):
    model: str | None = None
    prompt: str | None = None
    messages: list[ChatMessage] | None = None


class DetokenizeRequest(BaseModel):
    model: str | None = None
    tokens: list[int]


def _usage(prompt: int, completion: int) -> dict:
    return {"prompt_tokens": prompt, "completion_tokens": completion, "total_tokens": prompt + completion}


def build_app(driver, tokenizer, served_model_name: str, max_model_len: int, metrics=None) -> FastAPI:
    app = FastAPI(title="k8v4_xpu_b200")
    eos = getattr(tokenizer, "eos_token_id", None)

    def refuse_unsupported(req: _Common) -> None:
        if req.best_of is not None and not req.n <= req.best_of <= 16:
            raise HTTPException(400, "best_of must lie in [n, 16]")
        if req.best_of is not None and req.best_of > req.n and req.stream:
            raise HTTPException(400, "best_of above n is served without streaming")
        if req.use_beam_search:
            raise HTTPException(400, "beam search is not supported")
        if req.response_format and req.response_format.get("type", "text") != "text":
            raise HTTPException(400, "structured output (response_format) is not supported")
        if req.tools or req.guided_json is not None or req.guided_regex:
            raise HTTPException(400, "tool calls and JSON / regex guided decoding are not supported")
        if req.guided_choice is not None and (not req.guided_choice
                                              or not all(isinstance(c, str) and c for c in req.guided_choice)):
            raise HTTPException(400, "guided_choice takes a list of non-empty strings")

    def params_for(req: _Common, prompt_len: int) -> SamplingParams:
        refuse_unsupported(req)
        mt = req.max_completion_tokens if req.max_completion_tokens is not None else req.max_tokens
        mt = 16 if mt is None else mt  # an explicit 0 is refused below, not defaulted
        if mt == 0 and getattr(req, "echo", False):
            mt = 1  # echo only (prompt scoring): one token is generated and dropped
        elif mt < 1:
            raise HTTPException(400, "max_tokens must be positive")
        if prompt_len < 1:
            raise HTTPException(400, "empty prompt")
        if prompt_len + mt > max_model_len:
            raise HTTPException(400, "prompt (%d) + max_tokens (%d) exceeds max_model_len %d"
                                % (prompt_len, mt, max_model_len))
        stops = tuple(req.stop_token_ids) + ((eos,) if eos is not None else ())
        temperature = float(req.temperature or 0.0)
        top_p = 1.0 if req.top_p is None else float(req.top_p)
        top_k = 0 if req.top_k is None or req.top_k == -1 else int(req.top_k)
        if temperature < 0 or not 0.0 < top_p <= 1.0 or top_k < 0:
            raise HTTPException(400, "temperature must be >= 0, top_p in (0, 1], top_k >= 0 or -1")
        rep = 1.0 if req.repetition_penalty is None else float(req.repetition_penalty)
        pres = float(req.presence_penalty or 0.0)
        freq = float(req.frequency_penalty or 0.0)
        if rep <= 0 or not -2.0 <= pres <= 2.0 or not -2.0 <= freq <= 2.0:
            raise HTTPException(400, "repetition_penalty must be > 0; presence / frequency penalties in [-2, 2]")
        min_p = float(req.min_p or 0.0)
        min_tokens = int(req.min_tokens or 0)
        try:
            bias = {int(t): float(v) for t, v in (req.logit_bias or {}).items()}
        except ValueError:
            raise HTTPException(400, "logit_bias maps token ids to numbers")
        if not 0.0 <= min_p <= 1.0 or not 0 <= min_tokens <= mt or any(not -100 <= v <= 100 for v in bias.values()):
            raise HTTPException(400, "min_p in [0, 1], min_tokens in [0, max_tokens], logit_bias values in [-100, 100]")
        return SamplingParams(max_tokens=mt, ignore_eos=req.ignore_eos, stop_token_ids=stops,
                              temperature=temperature, top_p=top_p, top_k=top_k, seed=req.seed,
                              repetition_penalty=rep, presence_penalty=pres, frequency_penalty=freq,
                              min_p=min_p, logit_bias=bias or None, min_tokens=min_tokens,
                              allowed_sequences=(tuple(tuple(tokenizer.encode(c)) for c in req.guided_choice)
                                                 if req.guided_choice else None))

    async def run(prompt: list[int], params: SamplingParams):
        loop = asyncio.get_running_loop()
        out: asyncio.Queue = asyncio.Queue()
        try:
            h = driver.submit(prompt, params, loop, out)
        except RuntimeError as e:
            raise HTTPException(503, str(e))
        return h, out

    @app.get("/health")
    async def health():
        if not driver.healthy:
            return JSONResponse({"status": "error", "detail": (driver.error or "engine stopped")[-2000:]},
                                status_code=503)
        return {"status": "ok"}

    @app.get("/ping")
    async def ping():
        return await health()

    @app.get("/version")
    async def version():
        from .. import __version__
        return {"version": __version__}

    @app.post("/tokenize")
    async def tokenize(req: TokenizeRequest):
        """Token ids of a prompt, or of chat messages through the chat template."""
        if (req.prompt is None) == (req.messages is None):
            raise HTTPException(400, "give either prompt or messages")
        ids = (tokenizer.encode(req.prompt) if req.prompt is not None
               else tokenizer.apply_chat_template([m.model_dump() for m in req.messages]))
        return {"tokens": ids, "count": len(ids), "max_model_len": max_model_len}

    @app.post("/detokenize")
    async def detokenize(req: DetokenizeRequest):
        return {"prompt": tokenizer.decode(req.tokens)}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": served_model_name, "object": "model", "created": 0,
                                            "owned_by": "k8v4_xpu_b200", "max_model_len": max_model_len}]}

    @app.get("/metrics")
    async def metrics_ep():
        body = metrics.render() if metrics is not None else b""
        return Response(body, media_type=CONTENT_TYPE_LATEST)

    async def generate(prompt: list[int], req: _Common, chat: bool, request: Request):
        params = params_for(req, len(prompt))
        if not 1 <= req.n <= 16:
            raise HTTPException(400, "n must lie in [1, 16]")
        if chat:
            n_lp = int(req.top_logprobs or 0) if req.logprobs else None
        else:
            n_lp = None if req.logprobs is None or req.logprobs is False else int(req.logprobs)
        if n_lp is not None:
            if not 0 <= n_lp <= 20:
                raise HTTPException(400, "logprobs / top_logprobs must lie in [0, 20]")
            params = dataclasses.replace(params, logprobs=n_lp)
        echo = bool(getattr(req, "echo", False))
        echo_only = echo and (req.max_completion_tokens if req.max_completion_tokens is not None
                              else req.max_tokens) == 0
        if echo_only and req.stream:
            raise HTTPException(400, "max_tokens 0 with echo (prompt scoring) is served without streaming")
        if echo and n_lp is not None:
            params = dataclasses.replace(params, prompt_logprobs=n_lp)
        prompt_text = tokenizer.decode(prompt) if echo else ""

        def echo_part(h):
            """(tokens, entries) of the echoed prompt: the prompt's log-probabilities
            the engine recorded during prefill (the first token has none)."""
            seq = h.seq
            lps = list(getattr(seq, "prompt_logprobs", None) or []) if seq is not None else []
            return list(prompt), lps[:len(prompt)]

        def tok_str(t: int) -> str:
            return tokenizer.decode([int(t)])

        def lp_object(toks, lps, offset: int = 0):
            """The OpenAI logprobs object of ``toks`` (None when not asked for)."""
            if n_lp is None:
                return None
            lps = list(lps or []) + [None] * (len(toks) - len(lps or []))
            if chat:
                content = []
                for t, e in zip(toks, lps):
                    s = tok_str(t)
                    top = [{"token": tok_str(i), "logprob": v, "bytes": list(tok_str(i).encode("utf-8"))}
                           for i, v in (e[1] if e else [])]
                    content.append({"token": s, "logprob": e[0] if e else None, "bytes": list(s.encode("utf-8")),
                                    "top_logprobs": top})
                return {"content": content}
            tokens = [tok_str(t) for t in toks]
            offsets = []
            for s in tokens:
                offsets.append(offset)
                offset += len(s)
            return {"tokens": tokens, "token_logprobs": [e[0] if e else None for e in lps],
                    "top_logprobs": [({tok_str(i): v for i, v in e[1]} if e else None) for e in lps],
                    "text_offset": offsets}
        # n choices are n engine requests over the same prompt (the prefix
        # cache shares its pages); seeded requests give choice i seed + i
        # best_of candidates (n when unset) run as engine requests; the n with
        # the highest cumulative log-probability come back
        n_run = max(req.n, req.best_of or req.n)
        rank_by_lp = n_run > req.n
        if rank_by_lp and params.logprobs is None:
            params = dataclasses.replace(params, logprobs=0)  # the chosen tokens' entries rank the candidates
        runs = []
        for i in range(n_run):
            p = params if i == 0 else dataclasses.replace(
                params, seed=None if params.seed is None else params.seed + i)
            runs.append(await run(prompt, p))
        rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:24]
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        opts = req.stream_options or StreamOptions()

        def abort_all():
            for h, _ in runs:
                driver.abort(h)

        if not req.stream:
            async def collect(h, out):
                toks: list[int] = []
                all_lps: list = []
                reason = None
                matcher = StopMatcher(req.stop, req.include_stop_str_in_output)
                detok = IncrementalDecoder(tokenizer)
                parts: list[str] = []
                while True:
                    new, fin, why, lps = await out.get()
                    toks.extend(new)
                    all_lps.extend(lps or [None] * len(new))
                    if matcher.stops and not (fin and why and (why == "error" or why.startswith("rejected: "))):
                        shown, stopped = matcher.feed(detok.push(new, final=fin), final=fin)
                        parts.append(shown)
                        if stopped:  # a stop string ends the request: the engine drops the sequence
                            if not fin:
                                driver.abort(h)
                            reason = "stop"
                            break
                    if fin:
                        reason = why
                        break
                text = "".join(parts) if matcher.stops else tokenizer.decode(toks)
                return toks, text, reason, all_lps

            results = await asyncio.gather(*(collect(h, out) for h, out in runs))
            for _, _, reason, _ in results:
                if reason == "error":
                    raise HTTPException(500, "engine failed")
                if reason and reason.startswith("rejected: "):
                    raise HTTPException(400, reason[len("rejected: "):])
            if echo_only:  # prompt scoring: the one generated token is dropped
                results = [([], "", "length", []) for _ in results]
            usage = _usage(len(prompt), sum(len(r[0]) for r in results))
            if rank_by_lp:
                order = sorted(range(len(results)),
                               key=lambda j: -sum(e[0] for e in results[j][3] if e is not None))
                results = [results[j] for j in order[:req.n]]
                runs = [runs[j] for j in order[:req.n]]
            choices = []
            for i, (toks, text, reason, lps) in enumerate(results):
                if echo:
                    ptoks, plps = echo_part(runs[i][0])
                    plps = plps + [None] * (len(ptoks) - len(plps))
                    text, lp_toks, lps = prompt_text + text, ptoks + toks, plps + list(lps)
                else:
                    lp_toks = toks
                choice = ({"index": i, "message": {"role": "assistant", "content": text}, "finish_reason": reason}
                          if chat else {"index": i, "text": text, "finish_reason": reason, "logprobs": None})
                if n_lp is not None:
                    choice["logprobs"] = lp_object(lp_toks, lps)
                choice["token_ids"] = toks
                choices.append(choice)
            return {"id": rid, "object": obj, "created": created, "model": served_model_name,
                    "choices": choices, "usage": usage}

        async def events():
            n_out = 0
            chunk_obj = "chat.completion.chunk" if chat else "text_completion"
            merged: asyncio.Queue = asyncio.Queue()

            async def pump(i, out):
                while True:
                    item = await out.get()
                    await merged.put((i, item))
                    if item[1]:
                        return

            pumps = [asyncio.ensure_future(pump(i, out)) for i, (_, out) in enumerate(runs)]
            detoks = [IncrementalDecoder(tokenizer) for _ in runs]
            offsets = [0] * len(runs)  # text offsets of the completions logprobs
            echoed = [not echo] * len(runs)
            matchers = [StopMatcher(req.stop, req.include_stop_str_in_output) for _ in runs]
            live = set(range(len(runs)))
            if chat:
                for i in range(len(runs)):
                    first = {"id": rid, "object": chunk_obj, "created": created, "model": served_model_name,
                             "choices": [{"index": i, "delta": {"role": "assistant", "content": ""},
                                          "finish_reason": None}]}
                    if opts.continuous_usage_stats:
                        first["usage"] = _usage(len(prompt), 0)
                    yield "data: %s\n\n" % json.dumps(first)
            try:
                while live:
                    if await request.is_disconnected():
                        abort_all()
                        return
                    i, (new, fin, why, lps) = await merged.get()
                    if i not in live:
                        continue
                    if fin and why and why.startswith("rejected: "):
                        yield "data: %s\n\n" % json.dumps({"error": {"message": why[len("rejected: "):],
                                                                      "type": "invalid_request_error"}})
                        abort_all()
                        break
                    if not echoed[i]:  # the prompt goes out first, once the prefill has scored it
                        echoed[i] = True
                        ptoks, plps = echo_part(runs[i][0])
                        ch = {"index": i, "text": prompt_text, "finish_reason": None, "logprobs": None}
                        if n_lp is not None:
                            ch["logprobs"] = lp_object(ptoks, plps)
                            offsets[i] += len(prompt_text)
                        yield "data: %s\n\n" % json.dumps({"id": rid, "object": chunk_obj, "created": created,
                                                            "model": served_model_name, "choices": [ch]})
                    n_out += len(new)
                    text, stopped = matchers[i].feed(detoks[i].push(new, final=fin), final=fin)
                    if stopped and not fin:  # a stop string ends this choice here
                        driver.abort(runs[i][0])
                        fin, why = True, "stop"
                    elif stopped:
                        why = "stop"
                    if new or fin:
                        ch = ({"index": i, "delta": {"content": text}, "finish_reason": why if fin else None}
                              if chat else {"index": i, "text": text, "finish_reason": why if fin else None,
                                            "logprobs": None})
                        ch["token_ids"] = list(new)
                        if n_lp is not None:
                            ch["logprobs"] = lp_object(list(new), lps, offsets[i])
                            offsets[i] += sum(len(tok_str(t)) for t in new)
                        body = {"id": rid, "object": chunk_obj, "created": created, "model": served_model_name,
                                "choices": [ch]}
                        if opts.continuous_usage_stats:
                            body["usage"] = _usage(len(prompt), n_out)
                        yield "data: %s\n\n" % json.dumps(body)
                    if fin:
                        live.discard(i)
                if opts.include_usage:
                    yield "data: %s\n\n" % json.dumps({"id": rid, "object": chunk_obj, "created": created,
                                                       "model": served_model_name, "choices": [],
                                                       "usage": _usage(len(prompt), n_out)})
                yield "data: [DONE]\n\n"
            except asyncio.CancelledError:
                abort_all()
                raise
            finally:
                for t in pumps:
                    t.cancel()

        return StreamingResponse(events(), media_type="text/event-stream")

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest, request: Request):
        if isinstance(req.prompt, str):
            prompt = tokenizer.encode(req.prompt)
        elif req.prompt and isinstance(req.prompt[0], str):
            if len(req.prompt) != 1:
                raise HTTPException(400, "one prompt per request")
            prompt = tokenizer.encode(req.prompt[0])
        else:
            prompt = [int(t) for t in req.prompt]
        return await generate(prompt, req, False, request)

    @app.post("/v1/chat/completions")
    async def chat(req: ChatRequest, request: Request):
        prompt = tokenizer.apply_chat_template([m.model_dump() for m in req.messages])
        return await generate(prompt, req, True, request)

    return app
