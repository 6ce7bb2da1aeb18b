"""Multi-turn token traces and their conversion to training samples.

Reference counterparts: ``TokenTrace`` (``axrl/data/token_trace.py:38-273``),
``RolloutTrace`` (``axrl/data/rollout_trace.py:36-540``) and
``pack_rollout_traces_for_train_batches`` (:551-582).

A trace is a list of typed chunks (``init`` prompt, ``assistant`` model output with its
sampled logprobs, ``assistant_boundary``, ``tool_result``, ``user``).  Each assistant
turn yields one *turn sample*: the whole stream up to and including that turn, with
loss only on that turn's tokens (labels left-shifted by one).  Turn samples of one
trajectory share prefixes; :meth:`RolloutTrace.to_packed_samples` greedily groups
consecutive turns into label-aware prefix-tree merged samples of bounded length.

R3 bookkeeping: every assistant chunk may carry a routing handle covering the rows
captured for it; a path of ``n`` tokens has ``n - 1`` routing rows (row ``k`` routes the
token that predicts position ``k + 1``).  Compaction rewrites old tool results and keeps
only the routing handles that still describe a valid prefix.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Literal

import numpy as np

from axrl_b200.configs import IGNORE_INDEX
from axrl_b200.data.prefix_tree import MergingTree, merge_trajectory_samples
from axrl_b200.data.sample import Sample

ChunkType = Literal["init", "assistant", "assistant_boundary", "tool_result", "user"]


@dataclass
class TokenInfo:
    tokens: np.ndarray
    token_type: ChunkType
    logprobs: np.ndarray

    def __post_init__(self) -> None:
        self.tokens = np.asarray(self.tokens, dtype=np.int32)
        self.logprobs = np.asarray(self.logprobs, dtype=np.float32)


@dataclass
class TokenTrace:
    token_infos: list[TokenInfo] = field(default_factory=list)
    routing_handles: list[Any] = field(default_factory=list)
    token_info_index_per_handle: list[int] = field(default_factory=list)
    routing_row_count_per_handle: list[int] = field(default_factory=list)
    _turn_rewards: dict[int, float] = field(default_factory=dict, repr=False)

    # ---------------------------------------------------------------- flat views
    def _cat(self, parts: list[np.ndarray], dtype: Any) -> np.ndarray:
        return np.concatenate(parts).astype(dtype, copy=False) if parts else np.empty(0, dtype=dtype)

    @property
    def token_ids(self) -> np.ndarray:
        return self._cat([c.tokens for c in self.token_infos], np.int32)

    @property
    def token_count(self) -> int:
        return sum(len(c.tokens) for c in self.token_infos)

    @property
    def token_logprobs(self) -> np.ndarray:
        return self._cat([c.logprobs if len(c.logprobs) else np.zeros(len(c.tokens), np.float32) for c in self.token_infos], np.float32)

    @property
    def loss_mask(self) -> np.ndarray:
        return self._cat([np.full(len(c.tokens), c.token_type == "assistant") for c in self.token_infos], np.bool_)

    @property
    def turn_index(self) -> np.ndarray:
        out, k = [], 0
        for c in self.token_infos:
            if c.token_type == "assistant":
                out.append(np.full(len(c.tokens), k, np.int32))
                k += 1
            else:
                out.append(np.full(len(c.tokens), -1, np.int32))
        return self._cat(out, np.int32)

    @property
    def num_assistant_turns(self) -> int:
        return sum(c.token_type == "assistant" for c in self.token_infos)

    @property
    def captured_routing_rows(self) -> int:
        return sum(self.routing_row_count_per_handle)

    # ---------------------------------------------------------------- building
    def extend_tokens(self, new_tokens, logprobs=None, *, token_type: ChunkType, routing_handle=None, routing_row_count=None) -> None:  # noqa: ANN001
        new_tokens = np.asarray(new_tokens, dtype=np.int32)
        logprobs = np.zeros(len(new_tokens), np.float32) if logprobs is None else np.asarray(logprobs, np.float32)
        assert len(logprobs) == len(new_tokens)
        assert (token_type == "init") == (not self.token_infos), "the first chunk (and only it) is 'init'"
        if routing_handle is not None:
            assert token_type == "assistant", "routing handles belong to assistant chunks"
            if routing_row_count is None:
                routing_row_count = self.new_routing_row_count(len(new_tokens))
            self.routing_handles.append(routing_handle)
            self.token_info_index_per_handle.append(len(self.token_infos))
            self.routing_row_count_per_handle.append(int(routing_row_count))
        self.token_infos.append(TokenInfo(new_tokens, token_type, logprobs))

    def new_routing_row_count(self, new_token_count: int, *, prior_routing_rows: int | None = None) -> int:
        prior = self.captured_routing_rows if prior_routing_rows is None else prior_routing_rows
        rows = self.token_count + new_token_count - 1 - prior
        assert rows >= 0, "routing row count would be negative"
        return rows

    def set_turn_reward(self, turn_index: int, reward: float) -> None:
        assert 0 <= turn_index < self.num_assistant_turns
        self._turn_rewards[turn_index] = reward

    # ---------------------------------------------------------------- samples
    @staticmethod
    def _shift(v: np.ndarray, pad: Any) -> np.ndarray:
        return np.concatenate([v[1:], np.asarray([pad], dtype=v.dtype)]) if len(v) else v.copy()

    def _make_sample(self, loss_mask: np.ndarray, turn_index: np.ndarray, turn_reward: np.ndarray, max_length: int, pad_token_id: int) -> Sample:
        ids = self.token_ids
        n = len(ids)
        assert 0 < n <= max_length, f"trace length {n} exceeds max_length {max_length}"
        assert not bool(loss_mask[0]), "a trace must start with non-trainable context"
        lp = self.token_logprobs
        fields = dict(labels=self._shift(ids, IGNORE_INDEX), rollout_logprobs=self._shift(lp, 0.0), loss_mask=self._shift(loss_mask, False),
                      turn_index=self._shift(turn_index, -1), turn_reward=self._shift(turn_reward, 0.0))
        pad = max_length - n
        pads = dict(labels=IGNORE_INDEX, rollout_logprobs=0.0, loss_mask=False, turn_index=-1, turn_reward=0.0)
        if pad:
            ids = np.pad(ids, (0, pad), constant_values=pad_token_id)
            fields = {k: np.pad(v, (0, pad), constant_values=pads[k]) for k, v in fields.items()}
        return Sample(input_ids=ids, attention_mask=np.arange(max_length) < n, position_ids=np.arange(max_length), reward=0.0,
                      reward_baseline=0.0, advantage=np.zeros(max_length, np.float32),
                      routing_handles_per_path=[list(self.routing_handles)] if self.routing_handles else None, **fields)

    def to_last_turn_sample(self, max_length: int, pad_token_id: int) -> Sample:
        """Sample whose loss covers only the LAST (assistant) chunk."""
        last = self.token_infos[-1]
        assert last.token_type == "assistant"
        n = self.token_count
        lm = np.zeros(n, bool)
        ti = np.full(n, -1, np.int32)
        tr = np.zeros(n, np.float32)
        s = n - len(last.tokens)
        if len(last.tokens):
            lm[s:] = True
            ti[s:] = 0
            tr[s:] = self._turn_rewards.get(0, 0.0)
        return self._make_sample(lm, ti, tr, max_length, pad_token_id)

    def to_sample(self, max_length: int, pad_token_id: int) -> Sample:
        """Flat sample with every assistant chunk trainable."""
        ti = self.turn_index
        tr = np.asarray([self._turn_rewards.get(int(i), 0.0) if i >= 0 else 0.0 for i in ti], np.float32)
        return self._make_sample(self.loss_mask, ti, tr, max_length, pad_token_id)


class RolloutTrace:
    def __init__(self, max_length: int = 32768, pad_token_id: int = 0, assistant_boundary_token_id: int | None = None) -> None:
        self.max_length = max_length
        self.pad_token_id = pad_token_id
        self.boundary = assistant_boundary_token_id
        self.token_trace = TokenTrace()
        self.turn_samples: list[Sample] = []
        self.trajectory_id = -1

    def initialize(self, prompt_ids) -> None:  # noqa: ANN001
        assert not self.token_trace.token_infos, "trace already initialised"
        self.token_trace.extend_tokens(np.asarray(prompt_ids), token_type="init")

    @property
    def running_len(self) -> int:
        return self.token_trace.token_count

    @property
    def token_ids(self) -> np.ndarray:
        return self.token_trace.token_ids

    @property
    def routing_handles(self) -> list:
        return list(self.token_trace.routing_handles)

    def append_assistant(self, output_ids, output_logprobs, routing_handle=None, routing_row_count=None) -> None:  # noqa: ANN001
        """Append one model turn and record its per-turn training sample."""
        tt = self.token_trace
        tt.extend_tokens(np.asarray(output_ids), np.asarray(output_logprobs), token_type="assistant", routing_handle=routing_handle,
                         routing_row_count=routing_row_count)
        self.turn_samples.append(tt.to_last_turn_sample(tt.token_count, self.pad_token_id))
        ids = np.asarray(output_ids)
        if self.boundary is not None and (len(ids) == 0 or int(ids[-1]) != self.boundary):
            tt.extend_tokens(np.asarray([self.boundary]), token_type="assistant_boundary")

    def append_assistant_message(self, generation_output) -> None:  # noqa: ANN001
        self.append_assistant(generation_output.output_ids, generation_output.output_logprobs,
                              getattr(generation_output, "routing_handle", None))

    def append_user_or_tool_message(self, token_ids, role: Literal["user", "tool_result"] = "tool_result") -> None:  # noqa: ANN001
        self.token_trace.extend_tokens(np.asarray(token_ids), token_type=role)

    def set_turn_reward(self, turn_index: int, reward: float) -> None:
        self.token_trace.set_turn_reward(turn_index, reward)
        s = self.turn_samples[turn_index]
        s.turn_reward = np.where(s.loss_mask, np.float32(reward), np.float32(0.0)).astype(np.float32)

    def to_sample(self) -> Sample:
        assert self.turn_samples, "no assistant turn"
        return merge_trajectory_samples(self.turn_samples)

    def to_packed_samples(self, max_pack_length: int, *, allow_prefix_sharing: bool = True) -> list[Sample]:
        """Greedy grouping of consecutive turns into merged samples of at most ``max_pack_length``."""
        assert self.turn_samples and max_pack_length > 0
        if not allow_prefix_sharing:
            return [self._flat_single_sample(max_pack_length)]
        out, group, tree = [], [], MergingTree()
        for s in self.turn_samples:
            if len(s.input_ids) > max_pack_length:
                raise ValueError(f"turn sample length {len(s.input_ids)} exceeds max_pack_length {max_pack_length}")
            if tree.get_packed_len_if_add_path(s.input_ids) <= max_pack_length:
                group.append(s)
                tree.add_path(s.input_ids)
                continue
            out.append(self._merge(group))
            group, tree = [s], MergingTree()
            tree.add_path(s.input_ids)
        out.append(self._merge(group))
        for o in out:
            o.trajectory_id = self.trajectory_id
        return out

    @staticmethod
    def _merge(group: list[Sample]) -> Sample:
        assert all(g.reward_baseline == group[0].reward_baseline for g in group), "normalise group rewards before packing"
        m = merge_trajectory_samples(group, align_size=1)
        m.reward, m.reward_baseline = group[0].reward, group[0].reward_baseline
        return m

    def _flat_single_sample(self, max_pack_length: int) -> Sample:
        last = self.turn_samples[-1].input_ids
        for s in self.turn_samples[:-1]:
            assert np.array_equal(last[: len(s.input_ids)], s.input_ids), "flat export needs a linear prefix chain"
        s = self.token_trace.to_sample(len(last), self.pad_token_id)
        assert len(s.input_ids) <= max_pack_length
        # carry per-turn advantages (set on turn samples) onto the flat layout
        adv = np.zeros(len(s.input_ids), np.float32)
        for t in self.turn_samples:
            adv[: len(t.advantage)] = np.where(t.loss_mask, t.advantage, adv[: len(t.advantage)])
        s.advantage = adv
        s.reward, s.reward_baseline, s.trajectory_id = self.turn_samples[0].reward, self.turn_samples[0].reward_baseline, self.trajectory_id
        return s

    # ---------------------------------------------------------------- compaction
    def compact(self, max_recent_tool_results: int, placeholder_ids) -> None:  # noqa: ANN001
        """Replace all but the last ``max_recent_tool_results`` tool results with placeholder tokens.

        Routing handles of assistant chunks that come after the first rewritten chunk no
        longer describe the new token stream (their rows were captured with different
        context), so they are dropped; earlier handles remain a valid prefix."""
        tt = self.token_trace
        tool_idx = [i for i, c in enumerate(tt.token_infos) if c.token_type == "tool_result"]
        old = tool_idx[: max(0, len(tool_idx) - max_recent_tool_results)]
        if not old:
            return
        first = None
        for i in old:
            ph = np.asarray(placeholder_ids, np.int32)
            if not np.array_equal(tt.token_infos[i].tokens, ph):
                tt.token_infos[i] = TokenInfo(ph, "tool_result", np.zeros(len(ph), np.float32))
                first = i if first is None else min(first, i)
        if first is None:
            return
        keep = [k for k, ci in enumerate(tt.token_info_index_per_handle) if ci < first]
        tt.routing_handles = [tt.routing_handles[k] for k in keep]
        tt.token_info_index_per_handle = [tt.token_info_index_per_handle[k] for k in keep]
        tt.routing_row_count_per_handle = [tt.routing_row_count_per_handle[k] for k in keep]


def pack_rollout_traces_for_train_batches(traces: list[RolloutTrace], max_pack_length: int, allow_prefix_sharing: bool = True) -> list[Sample]:
    """Pack every trace; samples keep their trace's trajectory id (so splits stay in one global batch)."""
    out: list[Sample] = []
    for i, t in enumerate(traces):
        if t.trajectory_id < 0:
            t.trajectory_id = i
        out.extend(t.to_packed_samples(max_pack_length, allow_prefix_sharing=allow_prefix_sharing))
    return out
