"""The cached rollout equals a full re-prefill of the history at every step
(the reference's act(), model/model_decision_transformer.py:526-548)."""
import pytest
import torch

from oracle.dt_ref import dt_param_shapes
from oracle.seeded import seeded_state_dict


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,fused", [(torch.float32, False), (torch.bfloat16, False), (torch.bfloat16, True)])
def test_cached_rollout_matches_reprefill(dtype, fused):
    """fused: every block on the fused kernels (RMSNorm + q|k|v + RoPE GEMM before the
    decode kernel, RMSNorm + SwiGLU GEMM, residual GEMMs), in the rollout and in the
    re-prefill alike."""
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT
    from rl_for_mario_b200.rollout import DTRollout

    cfg = DTConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2,
                   context_len=16, dropout=0.0)
    cfgd = {k: getattr(cfg, k) for k in ("state_shape", "act_dim", "max_ep_len", "context_len", "hidden_size",
                                         "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                                         "intermediate_size")}
    model = MarioDT(cfg)
    model.load_state_dict(seeded_state_dict(dt_param_shapes(cfgd), 9), strict=True)
    model = model.cuda().to(dtype).eval()
    if fused:
        model.fuse_norms()
    B, T = 6, 8
    g = torch.Generator().manual_seed(0)
    states = torch.randint(0, 256, (B, T, 4, 84, 84), generator=g, dtype=torch.uint8).cuda()
    rtg = (torch.rand(B, T, generator=g) * 3000).cuda()
    ts = (torch.randint(0, 4000, (B, 1), generator=g) + torch.arange(T)).cuda()
    ro = DTRollout(model, num_envs=B, max_steps=T, page_size=16)
    actions = torch.zeros(B, T, dtype=torch.long, device="cuda")
    agree, worst = 0, 0.0
    for t in range(T):
        a, logits = ro.step(states[:, t], rtg[:, t], ts[:, t])
        actions[:, t] = a
        with torch.no_grad():
            full = model(states[:, :t + 1], actions[:, :t + 1], rtg[:, :t + 1], ts[:, :t + 1]).action_logits[:, -1]
        worst = max(worst, (logits - full.float()).abs().max().item())
        agree += int((full.argmax(-1) == a).sum())
    tol = 2e-2 if dtype == torch.float32 else 8e-2
    assert worst < tol, f"cached vs re-prefill logits differ by {worst:.3e}"
    assert agree >= B * T - 1
    assert ro.cache.length == 3 * T - 1


@pytest.mark.gpu
@pytest.mark.parametrize("fused", [False, True])
def test_graph_replayed_rollout_equals_eager(fused):
    """graphs=True: episode 1 runs the step body eagerly on the static buffers,
    episode 2 captures one graph per step index and replays it, episode 3 only
    replays.  Episodes 2 and 3 reproduce episode 1 bit for bit (same kernels on
    the same buffers), and all three match the plain eager rollout (whose input
    views have other layouts, so library GEMMs may round differently) within bf16
    noise; host cache lengths follow."""
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT
    from rl_for_mario_b200.rollout import DTRollout

    cfg = DTConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2,
                   context_len=16, dropout=0.0)
    cfgd = {k: getattr(cfg, k) for k in ("state_shape", "act_dim", "max_ep_len", "context_len", "hidden_size",
                                         "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                                         "intermediate_size")}
    model = MarioDT(cfg)
    model.load_state_dict(seeded_state_dict(dt_param_shapes(cfgd), 9), strict=True)
    model = model.cuda().to(torch.bfloat16).eval()
    if fused:
        model.fuse_norms()
    B, T = 6, 8
    g = torch.Generator().manual_seed(1)
    states = torch.randint(0, 256, (B, T, 4, 84, 84), generator=g, dtype=torch.uint8).cuda()
    rtg = (torch.rand(B, T, generator=g) * 3000).cuda()
    ts = (torch.randint(0, 4000, (B, 1), generator=g) + torch.arange(T)).cuda()
    eager = DTRollout(model, num_envs=B, max_steps=T, page_size=16)
    graph = DTRollout(model, num_envs=B, max_steps=T, page_size=16, graphs=True)
    det = torch.backends.cudnn.deterministic
    torch.backends.cudnn.deterministic = True  # run-to-run identical library convolutions
    try:
        first = []
        for episode in range(3):
            eager.reset()
            graph.reset()
            for t in range(T):
                a_e, l_e = eager.step(states[:, t], rtg[:, t], ts[:, t])
                a_g, l_g = graph.step(states[:, t], rtg[:, t], ts[:, t])
                if episode == 0:
                    first.append((a_g.clone(), l_g.clone()))
                else:
                    assert torch.equal(l_g, first[t][1]), (episode, t, (l_g - first[t][1]).abs().max().item())
                    assert torch.equal(a_g, first[t][0])
                assert (l_e - l_g).abs().max().item() < 8e-2
                assert graph.cache.length == eager.cache.length
                graph.prev_action = eager.prev_action  # both continue from the same actions
    finally:
        torch.backends.cudnn.deterministic = det
    assert len(graph._graphs) == T
