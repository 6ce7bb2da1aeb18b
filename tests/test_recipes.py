"""Recipes: GSM8K (parquet + chat template + verifier) through the online loop, Search-R1 tool use
with the BM25 retriever, and the black-box agent through the OpenAI proxy (reference
``axis_recipe/*``)."""

import asyncio
import sys
import textwrap

import numpy as np
import pandas as pd
import torch

from axrl_b200.data.conversation import Conversation, GenerationOutput, Message
from axrl_b200.processor.tokenizer import ByteTokenizer, ChatTokenizer


class _Scripted:
    """Rollout worker stand-in that answers with scripted texts (byte tokens)."""

    def __init__(self, texts):  # noqa: ANN001
        self.texts, self.i, self.tok = list(texts), 0, ByteTokenizer()
        self.prompts = []

    async def generate(self, inp):  # noqa: ANN001
        self.prompts.append(np.asarray(inp.input_ids))
        t = self.texts[min(self.i, len(self.texts) - 1)]
        self.i += 1
        ids = np.asarray(self.tok.encode(t) + [ByteTokenizer.eos_id], dtype=np.int32)
        return GenerationOutput(session_id=inp.session_id, output_ids=ids, output_logprobs=-np.ones(len(ids), dtype=np.float32), output_text=t,
                                output_text_with_special_tokens=t, cached_tokens=0, finish_reason="stop", e2e_elapsed_seconds=0.0,
                                stop_reason=None, retry=0)


class _Runtime:
    def __init__(self, worker):  # noqa: ANN001
        self.rollout_worker = worker


def _cfg():
    from axrl_b200.pipeline.config import PipelineExperimentConfig

    c = PipelineExperimentConfig()
    c.train_sampling_config.max_total_tokens = 2048
    return c


def test_gsm8k_recipe_online_loop(tmp_path):
    from axrl_b200.models.qwen3 import Qwen3Config
    from axrl_b200.pipeline.controller import PipelineController
    from axrl_b200.recipe.gsm8k_recipe import Gsm8kRecipe

    rows = [{"question": f"What is {i} + {i}?", "answer": f"{i} plus {i} #### {2 * i}"} for i in range(6)]
    pd.DataFrame(rows).to_parquet(tmp_path / "train.parquet")
    c = _cfg()
    c.megatron_worker.global_batch_size = 8
    c.megatron_worker.model.seq_length = 256
    c.online_rl_train.num_rollouts_per_conversation = 4
    c.online_rl_train.model_sync_every_n_global_updates = 1
    c.online_rl_train.batch_rollout_for_n_global_updates = 1
    c.online_rl_train.max_global_updates = 1
    c.online_rl_train.filter_zero_std = False
    c.online_rl_train.checkpoint_every_n_global_updates = None
    c.train_sampling_config.max_new_tokens = 12
    c.train_sampling_config.max_total_tokens = 160
    c.rollout_worker.max_running_requests = 8
    c.controller.max_running_requests = 8
    recipe = Gsm8kRecipe(c, ChatTokenizer(ByteTokenizer()), train_path=str(tmp_path / "train.parquet"))
    assert recipe.score("so #### 4", "2 plus 2 #### 4") == 1.0 and recipe.score("#### 5", "#### 4") == 0.0
    mcfg = Qwen3Config(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=16)
    torch.manual_seed(0)
    ctl = PipelineController(c, recipe, device="cpu", model_cfg=mcfg)
    ctl.train_dataset = recipe.dataset
    out = asyncio.run(ctl.start())
    assert len(out["history"]) == 1 and np.isfinite(out["history"][0]["train/grad_norm"])


def test_search_r1_episode_with_bm25():
    from axrl_b200.datasets.base_dataset import BaseDataset
    from axrl_b200.recipe.search_r1_recipe import BM25Index, SearchR1Recipe, exact_match, parse_action

    idx = BM25Index(["Paris is the capital of France.", "Berlin is the capital of Germany.", "The Nile is a river in Africa."])
    assert idx.search("capital of France", 1) == ["Paris is the capital of France."]
    assert parse_action("x <search> q1 </search>") == ("search", "q1") and exact_match("The Paris", ["paris"]) == 1.0
    conv = Conversation(messages=[Message("user", "What is the capital of France?")], conversation_id="q0", extra={"answers": ["Paris"]})
    c = _cfg()
    recipe = SearchR1Recipe(c, ChatTokenizer(ByteTokenizer()), BaseDataset([conv]), idx)
    worker = _Scripted(["<search>capital of France</search>", "<answer>Paris</answer>"])
    res = asyncio.run(recipe.run_rollout(recipe.dataset.conversations[0], _Runtime(worker)))
    assert res.metric.score == 1.0 and res.metric.extra["num_searches"] == 1.0
    assert b"Paris is the capital" in bytes(t - 16 for t in worker.prompts[1] if 16 <= t < 272)  # observation reached the model
    lm = res.trace.to_sample().loss_mask
    assert 0 < lm.sum() < len(lm)  # assistant turns trained, prompt and observation not


def test_blackbox_agent_through_proxy(tmp_path):
    from axrl_b200.datasets.base_dataset import BaseDataset
    from axrl_b200.recipe.blackbox_recipe import BlackboxRecipe

    agent = tmp_path / "agent.py"
    agent.write_text(textwrap.dedent("""
        import os, requests
        base = os.environ["OPENAI_BASE_URL"]
        msgs = [{"role": "user", "content": open("task.txt").read()}]
        for _ in range(2):
            r = requests.post(base + "/chat/completions", json={"model": "m", "messages": msgs}, timeout=30).json()
            msgs.append(r["choices"][0]["message"])
            msgs.append({"role": "user", "content": "tool output: ok"})
        open("answer.txt", "w").write(msgs[-2]["content"])
    """))
    conv = Conversation(messages=[Message("user", "say done")], conversation_id="t0")

    def reward(workdir, rc, out, conv):  # noqa: ANN001
        return 1.0 if rc == 0 and (workdir / "answer.txt").read_text().strip() == "done" else 0.0

    async def go():
        recipe = BlackboxRecipe(_cfg(), ChatTokenizer(ByteTokenizer()), BaseDataset([conv]), f"{sys.executable} {agent}", reward)
        await recipe.start_services()
        try:
            return await recipe.run_rollout(conv, _Runtime(_Scripted(["thinking", "done"])))
        finally:
            await recipe.stop_services({})

    res = asyncio.run(go())
    assert res.metric.score == 1.0 and res.metric.num_turns == 2
    s = res.trace.to_sample()
    assert s.loss_mask.sum() == len("thinking") + 1 + len("done") + 1  # both completions (+eos) trained
