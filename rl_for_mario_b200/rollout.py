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
    """Cached rollout over a batch of environments on this rank's GPU.

    ``graphs=True`` replays each step's device work (embeddings, state
    encoder, every layer with its cache append and attention, action head) as
    one CUDA graph per step index, so a step costs the host one graph launch
    instead of dozens of kernel launches and Python wrappers.  The first
    episode after construction runs eagerly (it initialises every library and
    kernel for each step's shapes); the next one captures step t's graph at step
    t and replays it; later episodes only replay.  Cache lengths and the RoPE
    rows a step uses depend on the step index, hence one graph per index; the
    graphs share one memory pool and are always replayed in capture order.
    The all-gather of the logits, the action choice and the host's cache
    bookkeeping stay outside the graphs.  Inputs are copied into static
    buffers (``frame_buffer`` can be written in place by the environment to
    avoid the frame copy)."""

    def __init__(self, model: MarioDT, num_envs: int, max_steps: int, page_size: int = 64,
                 group=None, device: Optional[torch.device] = None, graphs: bool = False):
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
        self.max_steps = max_steps
        self.use_graphs = graphs
        self.episodes = 0
        self._graphs = {}   # step index -> (CUDAGraph, host cache lengths after the step)
        self._pool = None
        self._static = None

    def reset(self) -> None:
        self.cache.reset()
        self.prev_action = None
        self.prev_timestep = None
        if self.steps:
            self.episodes += 1
        self.steps = 0

    # ------------------------------------------------------------ graph mode
    def _static_buffers(self, states: Tensor):
        if self._static is None:
            cfg = self.model.config
            b, dev = self.local_envs, self.device
            self._static = {
                "states": torch.empty((b,) + tuple(states.shape[1:]), dtype=states.dtype, device=dev),
                "rtg": torch.empty(b, dtype=torch.float32, device=dev),
                "ts": torch.empty(b, dtype=torch.long, device=dev),
                "prev_action": torch.zeros(b, dtype=torch.long, device=dev),
                "prev_ts": torch.zeros(b, dtype=torch.long, device=dev),
                "logits": torch.empty(b, cfg.act_dim, dtype=torch.float32, device=dev),
            }
        return self._static

    @property
    def frame_buffer(self) -> Optional[Tensor]:
        """The static [b, C, H, W] frame input of graph mode (after the first step):
        an environment that writes its observations here saves the per-step copy."""
        return None if self._static is None else self._static["states"]

    def _body(self, st: dict, first: bool) -> None:
        """One step's device work on the static buffers; writes st["logits"]."""
        bb = self.model.model
        cfg = self.model.config
        ts = st["ts"].clamp(0, cfg.max_ep_len - 1)
        te = bb.embed_timestep(ts)
        se = bb.state_encoder(st["states"].unsqueeze(1))[:, 0] + te
        re = bb.embed_return(st["rtg"].view(-1, 1).to(bb.embed_return.weight.dtype)) + te
        toks = [re, se]
        if not first:
            ae = bb.embed_action(st["prev_action"].clamp(0, cfg.act_dim - 1)) + bb.embed_timestep(st["prev_ts"])
            toks.insert(0, ae)
        h = bb.embed_norm(torch.stack(toks, dim=1))
        st["logits"].copy_(self.step_tokens(h))

    def _step_graphed(self, states: Tensor, returns_to_go: Tensor, timesteps: Tensor) -> Tensor:
        st = self._static_buffers(states)
        if states.data_ptr() != st["states"].data_ptr():
            st["states"].copy_(states)
        st["rtg"].copy_(returns_to_go)
        st["ts"].copy_(timesteps)
        t = self.steps
        if self.episodes == 0:
            # First episode: eager, which also initialises every kernel and library.
            self._body(st, t == 0)
        elif t not in self._graphs:
            if self._pool is None:
                self._pool = torch.cuda.graph_pool_handle()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self._pool):
                self._body(st, t == 0)  # the Python side advances the host cache lengths here
            self._graphs[t] = (g, [layer.length for layer in self.cache.layers])
            g.replay()
        else:
            g, lengths = self._graphs[t]
            g.replay()
            for layer, n in zip(self.cache.layers, lengths):
                layer.length = n
        return st["logits"]

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
        if self.steps >= self.max_steps:
            raise ValueError(f"episode already has {self.max_steps} steps (reset() starts a new one)")
        ts = timesteps.clamp(0, cfg.max_ep_len - 1).long()
        if self.use_graphs:
            if self.steps > 0:
                # The previous step's action (possibly set by the caller) and timestep.
                st = self._static
                st["prev_action"].copy_(self.prev_action)
                st["prev_ts"].copy_(self.prev_timestep)
            logits_local = self._step_graphed(states, returns_to_go, ts)
        else:
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
