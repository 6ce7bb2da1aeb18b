"""HTTP generation service and client (token ids in, token-aligned logprobs out).

Reference: ``OAICompatibleGenerationClient`` (``axrl/worker/oai_client.py:23-289``) talking to an
engine's native ``/generate`` endpoint with unbounded exponential-backoff retries, including
input-logprob scoring (``max_new_tokens = 0`` is sent as 1 and the output discarded) used for OPD
teacher logprobs; and the standalone engine servers the reference launches for teachers
(``axrl/utils/sglang_launch_utils.py:222-286``).

:func:`create_generate_app` exposes a :class:`RolloutWorker` over HTTP;
:class:`GenerationClient` is the client side used by rollout code and OPD annotation.
"""

from __future__ import annotations

import asyncio
import logging
import time
from typing import Any

import numpy as np

from axrl_b200.configs import OAIClientConfig, SamplingConfig
from axrl_b200.data.conversation import GenerationInput, GenerationOutput

logger = logging.getLogger(__name__)


def create_generate_app(worker: Any, teacher_model: Any = None):  # noqa: ANN201
    from fastapi import FastAPI
    from fastapi.responses import JSONResponse

    app = FastAPI()

    @app.post("/generate")
    async def generate(body: dict) -> JSONResponse:
        sp = body.get("sampling_params", {}) or {}
        sc = SamplingConfig(temperature=float(sp.get("temperature", 1.0)), max_new_tokens=int(sp.get("max_new_tokens", 256)),
                            max_total_tokens=int(sp.get("max_total_tokens", 1 << 20)))
        inp = GenerationInput(session_id=str(body.get("rid", "http")), input_ids=np.asarray(body["input_ids"], np.int32), sampling_config=sc)
        out: GenerationOutput = await worker.generate(inp)
        meta: dict[str, Any] = {"finish_reason": {"type": out.finish_reason}, "cached_tokens": out.cached_tokens,
                                "output_token_logprobs": [[float(l), int(t)] for l, t in zip(out.output_logprobs, out.output_ids)]}
        if body.get("return_logprob") and body.get("logprob_start_len") is not None and teacher_model is not None:
            meta["input_token_logprobs"] = teacher_model(np.asarray(body["input_ids"]), int(body["logprob_start_len"]))
        return JSONResponse({"output_ids": out.output_ids.tolist(), "meta_info": meta})

    @app.get("/health")
    async def health() -> dict:
        return {"ok": True}

    return app


class GenerationClient:
    def __init__(self, config: OAIClientConfig) -> None:
        import httpx

        self.config = config
        limits = httpx.Limits(max_connections=config.max_connections, max_keepalive_connections=config.max_keepalive_connections)
        self.http = httpx.AsyncClient(base_url=config.base_url, timeout=config.request_timeout_seconds, limits=limits)

    async def _post(self, payload: dict) -> dict:
        """POST /generate with unbounded exponential backoff (transport errors and 5xx)."""
        sleep = self.config.retry_initial_sleep_seconds
        attempt = 0
        while True:
            try:
                r = await self.http.post("/generate", json=payload)
                if r.status_code < 500:
                    r.raise_for_status()
                    return r.json()
                logger.warning("generate: HTTP %d, retrying in %.1fs", r.status_code, sleep)
            except Exception as e:  # noqa: BLE001
                import httpx

                if isinstance(e, httpx.HTTPStatusError) and e.response.status_code < 500:
                    raise
                logger.warning("generate: %s, retrying in %.1fs (attempt %d)", type(e).__name__, sleep, attempt)
            attempt += 1
            await asyncio.sleep(sleep)
            sleep = min(self.config.retry_max_sleep_seconds, sleep * 2)

    async def generate(self, inp: GenerationInput) -> GenerationOutput:
        sc = inp.sampling_config or self.config.sampling_config
        t0 = time.time()
        payload = {"rid": inp.session_id, "input_ids": inp.input_ids.tolist(), "return_logprob": True,
                   "sampling_params": {"temperature": sc.temperature, "max_new_tokens": sc.max_new_tokens or 256}}
        data = await self._post(payload)
        lps = data["meta_info"]["output_token_logprobs"]
        return GenerationOutput(session_id=inp.session_id, output_ids=np.asarray(data["output_ids"]), output_logprobs=np.asarray([x[0] for x in lps]),
                                output_text="", output_text_with_special_tokens="", cached_tokens=int(data["meta_info"].get("cached_tokens", 0)),
                                finish_reason=data["meta_info"]["finish_reason"]["type"], e2e_elapsed_seconds=time.time() - t0,
                                stop_reason=None, retry=0)

    async def score(self, input_ids: list[int], start: int) -> np.ndarray:
        """Log-probs of ``input_ids[start+1:]`` under the served model (teacher scoring)."""
        data = await self._post({"input_ids": input_ids, "return_logprob": True, "logprob_start_len": start,
                                 "sampling_params": {"temperature": 1.0, "max_new_tokens": 1}})
        return np.asarray(data["meta_info"]["input_token_logprobs"], dtype=np.float32)

    async def close(self) -> None:
        await self.http.aclose()
