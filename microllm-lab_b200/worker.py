"""Message host over the CUDA decode engine, mirroring the reference's worker protocol
(engine/worker.js:16-200): ``{cmd: "load" | "generate" | "unload" | "ping"}`` in, ``{type: "loaded" |
"token" | "done" | "unloaded" | "pong" | "error"}`` out, through a ``post`` callable.

Kept from the reference:
  - load (engine/worker.js:34-139): ``modelId = msg.modelId || msg.dtype || msg.kind || "petitgpt"``; the
    previous engine is destroyed before the new one is built; the ``loaded`` reply carries modelId, dtype,
    backend, gpu {name, vendor, bytesAllocated, limits} and the model cfg.
  - generate (engine/worker.js:141-186): the user prompt is encoded with the card's chat template; the
    prompt is cut to ``max(1, maxSeq - maxNew - 4)`` ids keeping a leading BOS; eosId is -1 with
    ``opts.ignoreEos``, else the card's eosId, else EOS; one ``token`` reply per id with the engine's phase
    meta; the ``done`` reply's text drops a final EOS; ``tokPerS = n / (totalMs / 1000)`` over the whole
    call (prefill included).
  - dispatch (engine/worker.js:188-200): ``maxNewTokens || 64``; unknown commands are ignored; any
    exception becomes ``{type: "error", message, stack}``.

Differences, by design of this backend:
  - The engine is always the CUDA one (``backend: "cuda"``): there is no CPU or WASM path to fall back
    to, so ``preferGpu`` has no effect and a missing device is an ``error`` reply.
  - The tokenizer comes from ``load``'s ``tokenizerSpec`` (a tokenizer.json object, as in the reference),
    or from any object with ``encode_messages(messages, card) -> ids`` and
    ``decode(ids, skip_special=False) -> str`` given to the constructor or as ``load``'s ``tokenizer``.
    There is no fetch of a default tokenizer.json. Without a tokenizer, ``generate`` takes ``promptIds``
    (ids as they are, still truncated), and the text fields are None.
  - The ``token`` replies are posted while the device generates: the kernels publish every id into
    mapped host memory as it is chosen (mllm_generate_stream), in generation order.
  - ``opts.specK`` / ``opts.ngram`` turn on the on-device prompt-lookup speculation.
"""
from __future__ import annotations

import math
import time
import traceback

from .engine import SPECIAL


def _nullish(v, default):
    """JavaScript's ``v ?? default``: the default only for a missing (None) value."""
    return default if v is None else v


def _js_truthy(v) -> bool:
    """JavaScript truthiness: undefined/null, false, 0, NaN and "" are false; every object is true."""
    if v is None or v is False:
        return False
    if isinstance(v, (int, float)):
        return v == v and v != 0
    if isinstance(v, str):
        return v != ""
    return True


def _js_number(v) -> float:
    """JavaScript's numeric coercion of a message field (``maxNew - 4`` and ``i < maxNew`` coerce it)."""
    if isinstance(v, bool):
        return float(v)
    try:
        return float(v)
    except (TypeError, ValueError):
        return float("nan")


def _new_token_count(max_new: float) -> int:
    """Ids engine/infer.js:603-646 yields for a (possibly fractional) maxNewTokens: the prefill's id, then
    one per i = 1, 2, ... while i < maxNewTokens."""
    if max_new != max_new or max_new <= 1:
        return 1
    return int(math.ceil(max_new))


class DecodeWorker:
    def __init__(self, post, tokenizer=None, engine_factory=None, device: int = 0):
        self.post = post
        self.tokenizer = tokenizer
        self.engine_factory = engine_factory
        self.device = device
        self.engine = None
        self.backend = "none"
        self.model_id = None
        self.card = {}

    # ---- dispatch (engine/worker.js:188-200)
    def handle(self, m) -> None:
        m = m or {}
        try:
            cmd = m.get("cmd")
            if cmd == "load":
                self._load(m)
            elif cmd == "generate":
                # `maxNewTokens || 64`, then numeric as the reference's arithmetic makes it
                mx = m.get("maxNewTokens")
                self._generate(m.get("prompt"), _js_number(mx if _js_truthy(mx) else 64), m.get("opts") or {},
                               m.get("promptIds"))
            elif cmd == "unload":
                self._drop_engine()
                self.post({"type": "unloaded"})
            elif cmd == "ping":
                self.post({"type": "pong"})
        except Exception as e:  # every failure is reported as a message, as the reference's worker does
            self.post({"type": "error", "message": str(e) or type(e).__name__, "stack": traceback.format_exc()})

    def _drop_engine(self):
        eng, self.engine = self.engine, None
        self.backend = "none"
        if eng is not None:
            eng.destroy()

    def _make_engine(self, buffer):
        if self.engine_factory is not None:
            return self.engine_factory(buffer)
        from .engine import CudaPetitGPT
        return CudaPetitGPT(buffer, device=self.device)

    # ---- load (engine/worker.js:34-139)
    def _load(self, msg):
        model_id = msg.get("modelId") or msg.get("dtype") or msg.get("kind") or "petitgpt"
        self.card = msg.get("card") or {}
        self.model_id = model_id
        if msg.get("tokenizer") is not None:
            self.tokenizer = msg["tokenizer"]
        elif _js_truthy(msg.get("tokenizerSpec")):  # a tokenizer.json object, as engine/worker.js:40-41 takes
            from .tokenizer import Tokenizer
            self.tokenizer = Tokenizer(msg["tokenizerSpec"])
        self._drop_engine()
        buffer = msg.get("buffer")
        if buffer is None:
            raise ValueError("load: no model buffer")
        self.engine = self._make_engine(buffer)
        self.backend = "cuda"
        self.post({
            "type": "loaded",
            "modelId": model_id,
            "dtype": model_id,
            "backend": self.backend,
            "wasm": False,
            "gpu": {
                "name": getattr(self.engine, "deviceName", f"cuda:{self.device}"),
                "vendor": "NVIDIA",
                "bytesAllocated": self.engine.bytesAllocated,
                "limits": None,
            },
            "cfg": dict(self.engine.cfg),
        })

    def _prompt_ids(self, prompt, prompt_ids):
        if prompt_ids is not None:
            return [int(i) for i in prompt_ids]
        if self.tokenizer is None:
            raise ValueError("generate: no tokenizer loaded; pass promptIds")
        return list(self.tokenizer.encode_messages([{"role": "user", "content": prompt}], self.card))

    def _decode(self, ids, skip_special=False):
        return None if self.tokenizer is None else self.tokenizer.decode(ids, skip_special)

    # ---- generate (engine/worker.js:141-186)
    def _generate(self, prompt, max_new, opts, prompt_ids=None):
        if self.engine is None:
            raise RuntimeError("no model loaded")
        ids = self._prompt_ids(prompt, prompt_ids)
        max_seq = self.card.get("maxSeqLen") or self.engine.cfg.get("maxSeqLen") or 2048
        max_prompt = max(1, max_seq - max_new - 4) if max_new == max_new else float("nan")
        if len(ids) > max_prompt:  # false for NaN, as in JavaScript
            bos = _nullish(self.card.get("bosId"), SPECIAL["BOS"])
            has_bos = ids[0] == bos
            keep = max_prompt - (1 if has_bos else 0)
            start = int(len(ids) - keep)  # Array.prototype.slice truncates a fractional start
            tail = ids[start:] if start < len(ids) else []
            ids = [ids[0]] + tail if has_bos else tail
        eos_id = -1 if opts.get("ignoreEos") else _nullish(self.card.get("eosId"), SPECIAL["EOS"])
        t0 = time.perf_counter()

        def on_token(tok, meta):
            self.post({"type": "token", "id": int(tok), "piece": self._decode([int(tok)], True), **meta})

        result = self.engine.generate(ids, maxNewTokens=_new_token_count(max_new), eosId=eos_id, onToken=on_token,
                                      specK=int(opts.get("specK") or 0), ngram=int(opts.get("ngram") or 3))
        gen = list(result["generatedIds"])
        text = self._decode(gen[:-1] if gen and gen[-1] == eos_id else gen, True)
        raw = self._decode(gen)
        total_ms = (time.perf_counter() - t0) * 1e3
        n = len(gen) or 1
        self.post({
            "type": "done",
            "text": text,
            "raw": raw,
            "generatedIds": gen,
            "promptIds": ids,
            "stopReason": result["stopReason"],
            "ttftMs": result["ttftMs"],
            "totalMs": total_ms,
            "tokPerS": n / (total_ms / 1000) if total_ms > 0 else 0.0,
            "backend": self.backend,
            "dtype": self.model_id,
        })
