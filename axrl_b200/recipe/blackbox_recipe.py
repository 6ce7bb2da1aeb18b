"""Black-box agent RL: an external agent program (OpenHands-style harness, any OpenAI client)
drives the policy through the OpenAI-compatible proxy; the episode's token stream is recorded
from the proxied requests and trained on.

Reference: ``axis_recipe/blackbox_rl/train_blackbox_rl.py:130-290`` with ``blackbox_env.py`` /
``openhands_env.py`` (agent in an E2B sandbox, proxy sessions, reward from a verifier).  Here each
rollout opens a proxy session, starts ``agent_command`` through a runner (process group, cgroup or
remote sandbox) with ``OPENAI_BASE_URL`` pointing at the session, serves every chat request of the
session with the rollout engine (rendered with the chat template; the completion is what the
agent receives), and, once the agent exits, scores the episode with ``reward_fn(workdir, exit
code, output)``.  Every assistant completion is a trained turn; the messages the agent adds in
between (tool results, user turns) are untrained context.
"""

from __future__ import annotations

import asyncio
import os
import tempfile
from pathlib import Path
from typing import Any, Callable

import numpy as np

from axrl_b200.data.conversation import RolloutResult
from axrl_b200.data.rollout_trace import RolloutTrace
from axrl_b200.metrics.response_metric import ResponseMetric
from axrl_b200.openai_proxy.chat_adapter import OpenAIChatAdapter
from axrl_b200.openai_proxy.server import OpenAIProxyServer, OpenAIProxySessionRegistry
from axrl_b200.processor.tokenizer import ChatTokenizer
from axrl_b200.recipe.base_recipe import BaseRecipe
from axrl_b200.runner.base_runner import ProcessGroupRunner


class BlackboxRecipe(BaseRecipe):
    def __init__(self, config: Any, tokenizer: Any, dataset: Any, agent_command: str,
                 reward_fn: Callable[[Path, int, str, Any], float], runner_factory: Callable[[], Any] = ProcessGroupRunner,
                 episode_timeout_s: float = 600.0, api_key: str | None = None) -> None:
        super().__init__(config)
        self.tok = tokenizer if isinstance(tokenizer, ChatTokenizer) else ChatTokenizer(tokenizer)
        self.dataset = dataset
        self.agent_command, self.reward_fn, self.runner_factory = agent_command, reward_fn, runner_factory
        self.episode_timeout_s, self.api_key = episode_timeout_s, api_key
        self.registry = OpenAIProxySessionRegistry(request_timeout_seconds=episode_timeout_s)
        self.server: OpenAIProxyServer | None = None
        inner = getattr(self.tok, "tok", None)
        self.adapter = OpenAIChatAdapter(lambda msgs, tools, **kw: self.tok.render(msgs, tools), self.tok.decode,
                                         chat_template=getattr(inner, "chat_template", None) if isinstance(getattr(inner, "chat_template", None), str) else None,
                                         tool_call_parser=getattr(config, "tool_call_parser", None) or "auto",
                                         reasoning_parser=getattr(config, "reasoning_parser", None))

    async def start_services(self) -> dict[str, Any]:
        self.server = OpenAIProxyServer(self.registry, api_key=self.api_key)
        self.server.start(asyncio.get_running_loop())
        await self.server.wait_started()
        return {"proxy": self.server}

    async def stop_services(self, services: Any) -> None:
        if self.server is not None:
            await self.server.stop()

    async def _serve(self, sid: str, runtime: Any, trace: RolloutTrace, stats: dict) -> None:
        while True:
            req = await self.registry.wait_for_request(sid, timeout_seconds=None)
            try:
                gi = self.adapter.convert_request(req.body, sid, self.config.train_sampling_config)
            except ValueError as e:  # a request the rollout cannot honour: the agent gets a 400
                await self.registry.fail(req.request_id, str(e), status_code=400)
                continue
            ids = np.asarray(gi.input_ids)
            cur = trace.token_ids if trace.running_len else np.zeros(0, dtype=np.int32)
            if len(cur) == 0:
                trace.initialize(ids)
            elif len(ids) >= len(cur) and np.array_equal(ids[:len(cur)], cur):
                if len(ids) > len(cur):
                    trace.append_user_or_tool_message(ids[len(cur):], "tool_result")
            else:  # the agent rewrote its history: continue from the new prompt as untrained context
                stats["history_rewrites"] += 1
                trace.append_user_or_tool_message(ids, "tool_result")
            out = await runtime.rollout_worker.generate(gi)
            trace.append_assistant(out.output_ids, out.output_logprobs)
            stats["turns"] += 1
            stats["response_tokens"] += len(out.output_ids)
            stats["finish"] = out.finish_reason
            await self.registry.respond(req.request_id, self.adapter.build_response(out, len(ids), req.body))

    async def run_rollout(self, conversation: Any, runtime: Any) -> RolloutResult:
        sid = f"{conversation.extra.get('group_id', conversation.conversation_id)}-{conversation.extra.get('group_index', 0)}".replace("/", "_")
        await self.registry.create_session(sid)
        trace = RolloutTrace(max_length=self.config.train_sampling_config.max_total_tokens)
        stats = {"turns": 0, "response_tokens": 0, "finish": "stop", "history_rewrites": 0}
        server = asyncio.create_task(self._serve(sid, runtime, trace, stats))
        workdir = Path(tempfile.mkdtemp(prefix="axrl-bb-"))
        (workdir / "task.txt").write_text("\n".join(m.text() for m in conversation.messages))
        runner = self.runner_factory()
        env = f"OPENAI_BASE_URL={self.server.base_url(sid)} OPENAI_API_KEY={self.api_key or 'none'} "
        try:
            rc, output = await runner.run(env + self.agent_command, workdir, timeout_seconds=self.episode_timeout_s)
        except TimeoutError:
            rc, output = -1, "timeout"
        finally:
            server.cancel()
            await self.registry.close_session(sid)
        score = float(self.reward_fn(workdir, rc, output, conversation))
        if not trace.running_len:  # the agent never called the model: an empty episode
            trace.initialize(np.asarray([int(self.tok.eos_id)], dtype=np.int32))
        metric = ResponseMetric(score=score, response_length=stats["response_tokens"], prompt_length=0, finish_reason=stats["finish"],
                                num_turns=stats["turns"], extra={"agent_exit_code": float(rc), "history_rewrites": float(stats["history_rewrites"])})
        return RolloutResult(conversation=conversation, trace=trace, metric=metric)


def env_var_agent_command(python_file: str) -> str:
    """Command that runs a python agent file with this interpreter."""
    import sys

    return f"{sys.executable} {os.path.abspath(python_file)}"
