"""Synthetic multi-turn agentic GRPO step: tool-using trajectories, partial rollout across steps,
prefix-tree packing of whole groups.

Workload (one GPU's share; the reference's agentic recipes, ``axrl/pipeline/controller.py`` with
``RolloutTrace`` turns, ``axrl/data/rollout_trace.py``):

* trajectories come in groups of ``group_size`` that share one ``prefix_len``-token system/task
  prefix; each trajectory runs ``U[min_turns, max_turns]`` turns;
* a turn is a model action of ``U[action_min, action_max]`` generated tokens (forced through EOS)
  followed by a tool observation of ``U[obs_min, obs_max]`` random token ids; the context is
  capped at ``max_context`` tokens;
* the rollout advances every live trajectory one turn per round (one batched ``generate``; the
  engine's prefix cache re-uses each trajectory's earlier context), until ``groups_per_step``
  groups are complete; the other groups keep their turns and continue in the next step (partial
  rollout), re-prefilling their context under the new weights;
* training packs every turn of a completed group into prefix trees (shared prefix and earlier
  turns computed once, varlen block-mask attention over the tree ranges), with the loss on model
  tokens only, group-normalised rewards (token-presence rule), old log-probs recomputed, one
  optimizer step.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from axrl_b200.configs import GrpoTrainerConfig, MegatronWorkerConfig
from axrl_b200.data.prefix_tree import MergingTree, add_sample_to_merging_tree, get_packed_len_if_merge, merge_trajectory_samples
from axrl_b200.data.rollout_trace import RolloutTrace
from axrl_b200.data.sample import SampleBatch
from axrl_b200.models.qwen3 import Qwen3Config
from axrl_b200.pipeline.rewards import group_advantages
from axrl_b200.rollout.engine import GenRequest, RolloutEngine
from axrl_b200.train.engine import TrainEngine
from axrl_b200.trainer.grpo_trainer import GrpoTrainer
from axrl_b200.utils import iostats


@dataclass
class AgenticConfig:
    group_size: int = 8
    inflight_groups: int = 2
    groups_per_step: int = 1
    prefix_len: int = 2048
    min_turns: int = 8
    max_turns: int = 32
    action_min: int = 32
    action_max: int = 256
    obs_min: int = 64
    obs_max: int = 512
    max_context: int = 32768
    pack_len: int = 32768
    reward_token: int = 7
    eos_token_id: int = 0
    temperature: float = 1.0
    seed: int = 0
    use_cuda_graph: bool = True
    kv_gb: float | None = None
    extra: dict = field(default_factory=dict)


@dataclass
class _Traj:
    gid: int
    idx: int
    turns_left: int
    context: list[int]
    trace: RolloutTrace
    done: bool = False
    reward: float = 0.0


class SyntheticAgentic:
    def __init__(self, model_cfg: Qwen3Config, worker_cfg: MegatronWorkerConfig, grpo_cfg: GrpoTrainerConfig, ac: AgenticConfig,
                 device: str | torch.device = "cpu", train_engine: TrainEngine | None = None) -> None:
        self.ac = ac
        self.mcfg = model_cfg
        self.device = torch.device(device)
        self.train = train_engine or TrainEngine(worker_cfg, model_cfg, self.device)
        self.trainer = GrpoTrainer(grpo_cfg)
        self.rng = np.random.default_rng(ac.seed)
        n_seq = ac.inflight_groups * ac.group_size
        kv_tokens = n_seq * (ac.max_context + 64)
        if ac.kv_gb is not None:
            per_tok = 2 * model_cfg.num_hidden_layers * model_cfg.num_key_value_heads * model_cfg.head_dim * 2
            kv_tokens = min(kv_tokens, int(ac.kv_gb * (1 << 30)) // per_tok)
        cuda = self.device.type == "cuda"
        self.rollout = RolloutEngine(self.train.model, max_batch=n_seq, kv_tokens=kv_tokens, page_size=64, max_context=ac.max_context + 8,
                                     max_prefill_tokens=max(16384, ac.prefix_len), seed=ac.seed, use_cuda_graph=ac.use_cuda_graph and cuda,
                                     eos_token_id=ac.eos_token_id, kv_memory_saver=cuda)
        if cuda and self.train.optim is not None:
            self.train.release_grads_after_step = True
        self.pool: list[list[_Traj]] = []
        self._gid = 0
        self._rid = 0
        self.step_idx = 0

    # ------------------------------------------------------------------ rollout
    def _new_group(self) -> list[_Traj]:
        ac, V = self.ac, self.mcfg.vocab_size
        prefix = self.rng.integers(1, V, size=ac.prefix_len).tolist()
        g = []
        for i in range(ac.group_size):
            tr = RolloutTrace(max_length=ac.max_context + ac.action_max + 8)
            tr.initialize(np.asarray(prefix, np.int32))
            g.append(_Traj(self._gid, i, int(self.rng.integers(ac.min_turns, ac.max_turns + 1)), list(prefix), tr))
        self._gid += 1
        return g

    def _round(self, live: list[_Traj]) -> tuple[int, int]:
        """One turn for every live trajectory: action, then the tool observation (or the end)."""
        ac, V = self.ac, self.mcfg.vocab_size
        reqs = []
        for t in live:
            n = int(self.rng.integers(ac.action_min, ac.action_max + 1))
            n = max(1, min(n, ac.max_context - len(t.context)))
            self._rid += 1
            reqs.append(GenRequest(rid=f"a{self._rid}", prompt=list(t.context), max_new_tokens=n, temperature=ac.temperature,
                                   forced_len=n, forced_token=ac.eos_token_id, seed_stream=self._rid))
        gen = obs = 0
        for t, res in zip(live, self.rollout.generate(reqs)):
            t.trace.append_assistant(np.asarray(res.output_ids, np.int32), np.asarray(res.output_logprobs, np.float32))
            t.context += res.output_ids
            gen += len(res.output_ids)
            if ac.reward_token in res.output_ids:
                t.reward = 1.0
            t.turns_left -= 1
            room = ac.max_context - len(t.context) - ac.action_min
            if t.turns_left <= 0 or room < ac.obs_min:
                t.done = True
                continue
            k = int(min(self.rng.integers(ac.obs_min, ac.obs_max + 1), room))
            ob = self.rng.integers(1, V, size=k).tolist()
            t.trace.append_user_or_tool_message(np.asarray(ob, np.int32))
            t.context += ob
            obs += k
        return gen, obs

    # ------------------------------------------------------------------ packing
    def pack_group(self, group: list[_Traj]) -> list:
        """Every turn sample of the group, greedily grouped into prefix trees of at most pack_len."""
        adv, _, _ = group_advantages([t.reward for t in group])
        out, cur, tree = [], [], MergingTree()
        for t, a in zip(group, adv):
            for s in t.trace.turn_samples:
                s.reward = t.reward
                s.advantage = np.where(s.loss_mask, np.float32(a), np.float32(0.0)).astype(np.float32)
                if cur and get_packed_len_if_merge(tree, s) > self.ac.pack_len:
                    out.append(merge_trajectory_samples(cur, align_size=1 if self.device.type == "cpu" else 8))
                    cur, tree = [], MergingTree()
                cur.append(s)
                add_sample_to_merging_tree(tree, s)
        if cur:
            out.append(merge_trajectory_samples(cur, align_size=1 if self.device.type == "cpu" else 8))
        for i, s in enumerate(out):
            s.trajectory_id = group[0].gid * 1000 + i
        return out

    # ------------------------------------------------------------------ the step
    def run_step(self) -> dict:
        ac = self.ac
        io0 = iostats.snapshot()
        t0 = time.perf_counter()
        while len(self.pool) < ac.inflight_groups:
            self.pool.append(self._new_group())
        self.rollout.acquire_kv()
        rounds = gen = obs = 0
        while sum(all(t.done for t in g) for g in self.pool) < ac.groups_per_step:
            live = [t for g in self.pool for t in g if not t.done]
            a, b = self._round(live)
            gen, obs, rounds = gen + a, obs + b, rounds + 1
        self.rollout.release_kv()
        rollout_s = time.perf_counter() - t0
        done = [g for g in self.pool if all(t.done for t in g)][: ac.groups_per_step]
        self.pool = [g for g in self.pool if not any(g is d for d in done)]

        t1 = time.perf_counter()
        samples = [s for g in done for s in self.pack_group(g)]
        batch = SampleBatch.from_samples(samples)
        pack_s = time.perf_counter() - t1
        t2 = time.perf_counter()
        batch["old_logprobs"] = self.train.compute_logprobs(batch, ac.temperature)
        batch["ref_logprobs"] = batch["old_logprobs"]
        logprob_s = time.perf_counter() - t2
        t3 = time.perf_counter()
        metrics = self.train.train_step(batch, self.trainer, temperature=ac.temperature)
        train_s = time.perf_counter() - t3
        self.rollout.reset_prefix_cache()  # colocated weight sync: shared weights, stale cache
        self.step_idx += 1
        io1 = iostats.snapshot()
        packed = int(batch["seq_len"].sum())
        logical = sum(len(t.context) for g in done for t in g)
        return {**metrics, "rollout_s": rollout_s, "pack_s": pack_s, "logprob_s": logprob_s, "train_s": train_s, "rounds": rounds,
                "generated_tokens": gen, "observation_tokens": obs, "trained_tokens": packed, "trajectory_tokens": logical,
                "trajectories": sum(len(g) for g in done), "turns": sum(len(t.trace.turn_samples) for g in done for t in g),
                "carried_groups": len(self.pool), "h2d_bytes": io1[0] - io0[0], "d2h_bytes": io1[1] - io0[1]}
