"""Async rollout worker around :class:`RolloutEngine` (the engine-adapter layer).

Reference counterpart: ``SGLangWorker`` (``axrl/worker/sglang_worker.py:49-851``):

* ``generate(GenerationInput) -> GenerationOutput`` token-in/token-out with sampled logprobs;
* **partial rollout**: ``pause_generation`` aborts everything in flight; each aborted call
  keeps its partial tokens and, after ``resume_generation``, re-submits
  ``input_ids + output_ids`` with the remaining budget, concatenating outputs (reference
  :338-405, :710-726);
* routed-expert capture rows per call (R3) go to the tensor store as a handle;
* memory release / resume and weight updates.

The engine runs on a dedicated thread that owns the GPU work; coroutines submit requests
through a thread-safe inbox and await futures.  One thread stepping the engine keeps
continuous batching intact across every concurrent caller.

When the engine thread ends (``shutdown`` on any rank of a lockstep group, or an exception in
the engine), every request it still holds is aborted and returned with its partial output, and
every call that was not yet admitted resolves as an empty ``abort``; after an exception the
callers' futures carry the exception instead.  No ``generate`` call is left waiting.
"""

from __future__ import annotations

import asyncio
import itertools
import logging
import queue
import threading
import time
from typing import Any

import numpy as np

from axrl_b200.configs import SamplingConfig
from axrl_b200.data.conversation import GenerationInput, GenerationOutput
from axrl_b200.rollout.engine import GenRequest, GenResult, RolloutEngine

log = logging.getLogger(__name__)


class _DecodeOnly:
    """The tokenizer surface a grammar needs: ids -> text."""

    def __init__(self, fn: Any) -> None:
        self.decode = fn


class RolloutWorker:
    def __init__(self, engine: RolloutEngine, sampling: SamplingConfig | None = None, continue_after_abort: bool = True,
                 tensor_store: Any = None, eos_token_id: int | None = None, decode_fn: Any = None) -> None:
        self.engine = engine
        self.sampling = sampling or SamplingConfig()
        self.continue_after_abort = continue_after_abort
        self.store = tensor_store
        self.eos = eos_token_id
        self.decode_fn = decode_fn
        if decode_fn is not None and getattr(engine, "tokenizer", None) is None:
            engine.tokenizer = _DecodeOnly(decode_fn)  # token strings for tool-call grammars
        self._inbox: queue.Queue = queue.Queue()
        self._pending: dict[str, tuple[asyncio.AbstractEventLoop, asyncio.Future, int]] = {}
        self._lock = threading.Lock()  # guards _pending and _closed
        self._closed = False
        self._error: BaseException | None = None
        self._ready = threading.Event()
        self._ready.set()
        self._pause_req = threading.Event()
        self._stop = threading.Event()
        self._ids = itertools.count()
        self._thread = threading.Thread(target=self._run, name="rollout-engine", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------------ engine thread
    def _drain_inbox(self) -> None:
        try:
            while True:
                self.engine.add_requests([self._inbox.get_nowait()])
        except queue.Empty:
            pass

    def _loop_lockstep(self) -> None:
        """Engine thread of a data-parallel-attention engine: every rank's thread takes each decision
        together (one small all-reduce per iteration), so every rank steps, pauses and stops at the
        same iteration.  A pause happens once every rank asked for it; after it the thread waits for
        this rank's resume, and its next all-reduce waits for every rank's, so the engine's expert
        collectives never overlap a rank's training."""
        eng = self.engine
        while True:
            self._drain_inbox()
            work, not_paused, stop = eng._ep_max([int(bool(eng.waiting or eng.running)), int(not self._pause_req.is_set()),
                                                  int(self._stop.is_set())])
            if stop:
                return
            if not not_paused:  # every rank asked to pause
                for r in eng.abort_all():
                    self._resolve(r)
                self._pause_req.clear()
                while not self._ready.wait(0.05):
                    pass
                continue
            if not work:
                time.sleep(0.001)
                continue
            for r in eng.step():
                self._resolve(r)

    def _run(self) -> None:
        lockstep = getattr(self.engine, "dp_attention", False)
        try:
            self._loop_lockstep() if lockstep else self._loop()
        except BaseException as e:  # noqa: BLE001
            log.exception("rollout engine thread failed")
            self._error = e
            self._finish(e)
            if lockstep:
                # Best effort: tell the peers to stop at their next decision.  Peers that are inside
                # a forward waiting for this rank end through their own collective timeouts.
                try:
                    self.engine._ep_max([0, 1, 1])
                except Exception:  # noqa: BLE001
                    pass
            return
        self._finish(None)

    def _finish(self, exc: BaseException | None) -> None:
        """Resolve every call this worker still holds; later submissions are refused."""
        with self._lock:
            self._closed = True
        done: list[GenResult] = []
        try:
            done = self.engine.abort_all()
        except Exception:  # noqa: BLE001
            log.exception("abort_all failed while stopping the rollout engine")
        try:
            while True:  # admitted to the inbox but never to the engine
                r = self._inbox.get_nowait()
                done.append(GenResult(r.rid, [], [], "abort", len(r.prompt)))
        except queue.Empty:
            pass
        if exc is None:
            for r in done:
                self._resolve(r)
        with self._lock:
            rest, self._pending = self._pending, {}
        err = exc if exc is not None else None
        for rid, (loop, fut, plen) in rest.items():
            if err is not None:
                loop.call_soon_threadsafe(lambda f=fut, e=err: f.done() or f.set_exception(RuntimeError(f"rollout engine failed: {e!r}")))
            else:
                res = GenResult(rid, [], [], "abort", plen)
                loop.call_soon_threadsafe(lambda f=fut, r=res: f.done() or f.set_result(r))
        self._ready.set()  # wake callers waiting to resubmit

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                while True:
                    req = self._inbox.get_nowait()
                    self.engine.add_requests([req])
            except queue.Empty:
                pass
            if self._pause_req.is_set():
                for r in self.engine.abort_all():
                    self._resolve(r)
                self._pause_req.clear()
                continue
            if not (self.engine.waiting or self.engine.running):
                time.sleep(0.0005)
                continue
            for r in self.engine.step():
                self._resolve(r)

    def _resolve(self, res: GenResult) -> None:
        with self._lock:
            loop, fut, _ = self._pending.pop(res.rid, (None, None, 0))
        if fut is not None:
            loop.call_soon_threadsafe(lambda: fut.done() or fut.set_result(res))

    async def _submit(self, req: GenRequest) -> GenResult:
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        with self._lock:
            closed = self._closed
            if not closed:
                self._pending[req.rid] = (loop, fut, len(req.prompt))
                self._inbox.put(req)
        if closed:
            if self._error is not None:
                raise RuntimeError(f"rollout engine failed: {self._error!r}")
            return GenResult(req.rid, [], [], "abort", len(req.prompt))
        return await fut

    # ------------------------------------------------------------------ public API
    async def generate(self, inp: GenerationInput) -> GenerationOutput:
        sc = inp.sampling_config or self.sampling
        ids = [int(x) for x in np.asarray(inp.input_ids)]
        budget = sc.max_new_tokens if sc.max_new_tokens is not None else max(1, sc.max_total_tokens - len(ids))
        stop = (self.eos,) if self.eos is not None else ()
        out_ids: list[int] = []
        out_lps: list[float] = []
        retry = 0
        t0 = time.time()
        inp.event_timing.stamp("worker_received")
        routing = []
        from axrl_b200.rollout.grammar import tool_call_schema, tool_call_structural_tag

        schema = tool_call_schema(getattr(inp, "tools", None), getattr(inp, "tool_choice", None))
        tag = (tool_call_structural_tag(inp.tools, inp.tool_call_parser)
               if schema is None and inp.tools and inp.tool_choice in (None, "auto") else None)
        while True:
            await asyncio.get_running_loop().run_in_executor(None, self._ready.wait)
            rid = f"{inp.session_id}#{next(self._ids)}"
            req = GenRequest(rid=rid, prompt=ids + out_ids, max_new_tokens=budget - len(out_ids), temperature=sc.temperature,
                             stop_token_ids=stop, capture_routing=inp.capture_routing, top_k=sc.top_k, top_p=sc.top_p, min_p=sc.min_p,
                             presence_penalty=sc.presence_penalty, frequency_penalty=sc.frequency_penalty,
                             repetition_penalty=sc.repetition_penalty, json_schema=schema, structural_tag=tag, gen_prefix=tuple(out_ids))
            res = await self._submit(req)
            out_ids += res.output_ids
            out_lps += res.output_logprobs
            if res.routed_experts is not None:
                routing.append(res.routed_experts)
            if res.finish_reason != "abort" or not self.continue_after_abort or len(out_ids) >= budget or self._closed:
                break
            retry += 1
        handle = None
        if routing and self.store is not None:
            rows = np.concatenate(routing, 0)[inp.routed_expert_start_index:]
            handle = self.store.put(rows)
        inp.event_timing.stamp("worker_returned")
        text = self.decode_fn(out_ids) if self.decode_fn else ""
        return GenerationOutput(session_id=inp.session_id, output_ids=np.asarray(out_ids), output_logprobs=np.asarray(out_lps),
                                output_text=text, output_text_with_special_tokens=text, cached_tokens=res.cached_tokens,
                                finish_reason=res.finish_reason, e2e_elapsed_seconds=time.time() - t0, stop_reason=None, retry=retry,
                                routing_handle=handle, event_timing=inp.event_timing)

    def pause_generation(self) -> None:
        """Abort everything in flight; calls resume later from their partial outputs."""
        self._ready.clear()
        self._pause_req.set()
        while self._pause_req.is_set() and self._thread.is_alive():
            time.sleep(0.001)

    def resume_generation(self) -> None:
        self._ready.set()

    def release_memory(self) -> None:
        self.pause_generation()
        self.engine.reset_prefix_cache()

    def shutdown(self) -> None:
        self._stop.set()
        self._ready.set()
        self._thread.join(timeout=5)
