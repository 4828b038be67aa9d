"""KV-cached batched rollout of the Decision Transformer, single- and multi-GPU.

The reference's act() (model/model_decision_transformer.py:526-548) re-runs
the whole context every step.  Here every environment keeps a paged KV cache
and a step appends only the new tokens.  Because the action a_t is the
output of step t, step t appends (a_{t-1}, R_t, s_t): the cache then holds the
reference's interleaved sequence R_0 s_0 a_0 R_1 s_1 a_1 ... (:416-420), and
the logits of s_t (the state token, :505-506) equal those of a full re-prefill
of the history.  The loop structure follows the reference's batched PPO
rollout (trainer/train_ppo_finetune.py:397-437): policy -> actions for all
environments -> environment step.

Multi-GPU: environments are sharded into contiguous slices, one per rank
(rank r owns [r B/N, (r+1) B/N)); weights are replicated and the caches are
rank-local.  The only collective is an all-gather of the [B/N, act_dim]
action logits per step, so every rank holds the full action vector (the
reference steps all environments with one action array, :408).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .cache import PagedKVCache
from .dt_model import MarioDT

Tensor = torch.Tensor


def shard_range(num_envs: int, rank: int, world: int):
    """Contiguous slice [start, stop) of environments owned by `rank`."""
    if num_envs % world:
        raise ValueError(f"{num_envs} environments do not split evenly over {world} ranks")
    per = num_envs // world
    return rank * per, (rank + 1) * per


def gather_rows(local: Tensor, group=None) -> Tensor:
    """All-gathers equal [b, ...] row blocks of every rank into [world * b, ...] (rank order)."""
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return local
    world = dist.get_world_size(group)
    if world == 1:
        return local
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=0)


class DTRollout:
    """Cached rollout over a batch of environments on this rank's GPU."""

    def __init__(self, model: MarioDT, num_envs: int, max_steps: int, page_size: int = 64,
                 group=None, device: Optional[torch.device] = None):
        cfg = model.config
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None or (dist.is_available() and
                                                                           dist.is_initialized())) else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.num_envs = num_envs
        self.lo, self.hi = shard_range(num_envs, self.rank, self.world)
        self.local_envs = self.hi - self.lo
        self.device = device or next(model.parameters()).device
        attn0 = model.model.layers[0].self_attn
        kv_dtype = attn0.compute_dtype or next(model.parameters()).dtype
        max_len = 3 * max_steps
        if max_len > cfg.max_position_embeddings:
            raise ValueError(f"{max_steps} steps need {max_len} positions > {cfg.max_position_embeddings}")
        self.cache = PagedKVCache(cfg.num_hidden_layers, self.local_envs, cfg.num_key_value_heads,
                                  cfg.hidden_size // cfg.num_attention_heads, max_len, page_size, kv_dtype,
                                  self.device)
        self.prev_action: Optional[Tensor] = None
        self.prev_timestep: Optional[Tensor] = None
        self.steps = 0

    def reset(self) -> None:
        self.cache.reset()
        self.prev_action = None
        self.prev_timestep = None
        self.steps = 0

    @torch.no_grad()
    def step_tokens(self, tokens: Tensor) -> Tensor:
        """Runs [b, n, H] new token states (after embed_norm) through the layers with the
        cache; returns this rank's action logits from the last token, [b, act_dim]."""
        bb = self.model.model
        hidden, _ = bb.run_layers(tokens, None, self.cache, use_cache=True, flat=True)
        return self.model.action_head(hidden[:, -1])

    @torch.no_grad()
    def step(self, states: Tensor, returns_to_go: Tensor, timesteps: Tensor, deterministic: bool = True):
        """One environment step for this rank's environments.

        states [b, C, H, W] uint8, returns_to_go [b], timesteps [b] (b = local
        environments).  Returns (actions [B] for all environments, logits [B, act_dim]).
        """
        bb = self.model.model
        cfg = self.model.config
        ts = timesteps.clamp(0, cfg.max_ep_len - 1).long()
        te = bb.embed_timestep(ts)
        se = bb.state_encoder(states.unsqueeze(1))[:, 0] + te
        re = bb.embed_return(returns_to_go.view(-1, 1).to(bb.embed_return.weight.dtype)) + te
        toks = [re, se]
        if self.prev_action is not None:
            tp = bb.embed_timestep(self.prev_timestep)
            toks.insert(0, bb.embed_action(self.prev_action.clamp(0, cfg.act_dim - 1)) + tp)
        h = bb.embed_norm(torch.stack(toks, dim=1))
        logits_local = self.step_tokens(h)
        logits = gather_rows(logits_local.float(), self.group)
        if deterministic:
            actions = logits.argmax(-1)
        else:
            actions = torch.distributions.Categorical(logits=logits).sample()
        self.prev_action = actions[self.lo:self.hi]
        self.prev_timestep = ts
        self.steps += 1
        return actions, logits
