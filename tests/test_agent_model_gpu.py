"""The Llama-shaped model and the agent loop on small configurations.

Model parity: our forward (bf16 activations, cuBLAS GEMMs, sm_100a paged prefill / decode,
pool appends) against an fp32 torch restatement with the same weights and the CPU attention
oracle, for a prefill followed by teacher-forced decode steps.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import attention as ora
from loopfuse_b200.agent_loop import AgentLoop, AgentLoopConfig
from loopfuse_b200.llama import LlamaConfig, LlamaShaped
from loopfuse_b200.runtime.kv_pool import KVPool

pytestmark = pytest.mark.gpu

SMALL = LlamaConfig(d_model=256, layers=2, q_heads=4, kv_heads=2, head_dim=128, ffn=512, vocab=1000)


def _reference_logits(m: LlamaShaped, tokens: torch.Tensor) -> torch.Tensor:
    """fp32 restatement over the whole sequence; logits of the last position."""
    c = m.cfg
    T = tokens.numel()
    x = m.embed[tokens].float().cpu()
    pos = torch.arange(T).float()
    ang = pos[:, None] * m.inv_freq.cpu()[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]

    def rms(v, w):
        return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + c.eps) * w.float().cpu()

    def rope(v):
        h = v.shape[-1] // 2
        return torch.cat([v[..., :h] * cos - v[..., h:] * sin, v[..., h:] * cos + v[..., :h] * sin], -1)

    nq, nk = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
    for l in range(c.layers):
        h = rms(x, m.attn_norm[l])
        qkv = h @ m.wqkv[l].float().cpu()
        q = rope(qkv[:, :nq].view(T, c.q_heads, c.head_dim))
        k = rope(qkv[:, nq:nq + nk].view(T, c.kv_heads, c.head_dim))
        v = qkv[:, nq + nk:].view(T, c.kv_heads, c.head_dim)
        o, _ = ora.prefill(q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None], v.permute(1, 0, 2)[None])
        x = x + o[0].permute(1, 0, 2).reshape(T, nq) @ m.wo[l].float().cpu()
        h = rms(x, m.ffn_norm[l])
        gu = h @ m.w13[l].float().cpu()
        x = x + (F.silu(gu[:, :c.ffn]) * gu[:, c.ffn:]) @ m.w2[l].float().cpu()
    return (rms(x[-1:], m.final_norm) @ m.lm_head.float().cpu())[0]


def test_model_prefill_then_decode_matches_fp32_reference():
    m = LlamaShaped(SMALL, seed=1, std=0.05)
    pool = KVPool(num_layers=SMALL.layers, num_heads=SMALL.q_heads, num_kv_heads=SMALL.kv_heads,
                  head_dim=SMALL.head_dim, max_seq_len=256, max_slots=2, dtype=torch.bfloat16)
    s = pool.allocate_slot()
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, SMALL.vocab, (43,), generator=g)
    got = m.forward(toks[:40].cuda(), pool, [s], [40], return_logits=True)[0].cpu()
    for i in range(40, 43):                                   # teacher-forced decode
        ref = _reference_logits(m, toks[:i])
        cos = F.cosine_similarity(got, ref, dim=0).item()
        assert cos > 0.999, (i, cos)
        assert (got - ref).abs().max().item() < 0.1 * ref.abs().max().item()
        got = m.forward(toks[i:i + 1].cuda(), pool, [s], [1], return_logits=True)[0].cpu()


def test_small_agent_loop_completes_every_step():
    m = LlamaShaped(SMALL, seed=2)
    cfg = AgentLoopConfig(sessions=6, steps=2, prefix_tokens=64, question_tokens=16, decode_tokens=3,
                          tool_ms=5.0, tool_len_mean=10, tool_len_cap=20, spec_tokens=4, seed=3)
    st = AgentLoop(m, cfg).run()
    assert st.steps_done == cfg.sessions * cfg.steps
    assert st.decode_tokens >= cfg.sessions * cfg.steps * (cfg.decode_tokens - 1)
    assert st.steps_per_s > 0


def test_graphed_decode_matches_eager_decode():
    """Graph replays (padded batch buckets) advance the same sessions as eager forwards on the
    same input tokens: the same pool metadata, next tokens that agree (GEMMs of another batch
    size may round differently), the sessions' K/V within bf16 rounding."""
    from loopfuse_b200.llama import GraphedDecode
    m = LlamaShaped(SMALL, seed=4)
    runs = []
    for graphed in (False, True):
        pool = KVPool(num_layers=SMALL.layers, num_heads=SMALL.q_heads, num_kv_heads=SMALL.kv_heads,
                      head_dim=SMALL.head_dim, max_seq_len=512, max_slots=24, dtype=torch.bfloat16)
        root = pool.alloc()
        g = torch.Generator().manual_seed(5)
        m.forward(torch.randint(0, SMALL.vocab, (64,), generator=g).cuda(), pool, [root], [64])
        ss = pool.fork(root, 64, n=20)
        lens = [int(x) for x in torch.randint(1, 40, (20,), generator=g)]
        m.forward(torch.randint(0, SMALL.vocab, (sum(lens),), generator=g).cuda(), pool, ss, lens,
                  n_prefix_pages=4)
        pad = pool.pad_session(root, 64)
        gd = GraphedDecode(m, pool, pad, n_prefix_pages=4) if graphed else None
        outs = []
        for it in range(6):
            batch = ss[: 20 - 3 * it]                        # shrinking batch: 20, 17, ..., 5
            tb = [int(x) for x in torch.randint(0, SMALL.vocab, (len(batch),), generator=g)]
            if graphed:
                nxt = gd.step(batch, tb)[: len(batch)].tolist()
                gd.raise_if_failed()
            else:
                nxt = m.forward(torch.tensor(tb, device="cuda"), pool, batch, [1] * len(batch),
                                n_prefix_pages=4).tolist()
            outs.append(nxt)
        snap = pool.snapshot()
        kv = [torch.cat([pool.read(st, l)[0] for l in range(SMALL.layers)]) for st in ss]
        runs.append((outs, snap, [st.current_len for st in ss], kv))
    (o_e, s_e, l_e, k_e), (o_g, s_g, l_g, k_g) = runs
    assert l_e == l_g
    assert s_e["block_table"] == s_g["block_table"] and s_e["seq_len"] == s_g["seq_len"]
    assert s_e["free_queue"] == s_g["free_queue"] and s_e["refcount"] == s_g["refcount"]
    flat_e = [t for o in o_e for t in o]
    flat_g = [t for o in o_g for t in o]
    assert sum(a == b for a, b in zip(flat_e, flat_g)) >= 0.9 * len(flat_e)
    for a, b in zip(k_e, k_g):                                # the sessions' own K, every layer
        assert (a.float() - b.float()).abs().max().item() < 0.05


def test_agent_loop_speculation_changes_no_session_length_and_returns_every_page():
    """Speculative prefill of the observation template in idle windows moves work earlier but
    not its amount: with speculation on and off every session ends with the same number of
    tokens (prompt, questions, templates, tool outputs, decoded tokens), and after the loop
    every page except the system prompt's is back in the free queue."""
    m = LlamaShaped(SMALL, seed=6)
    runs = {}
    for spec in (True, False):
        cfg = AgentLoopConfig(sessions=8, steps=3, prefix_tokens=64, question_tokens=16,
                              decode_tokens=4, tool_ms=20.0, tool_len_mean=12, tool_len_cap=30,
                              spec_tokens=4, speculative=spec, seed=7)
        loop = AgentLoop(m, cfg)
        st = loop.run()
        assert st.steps_done == cfg.sessions * cfg.steps
        runs[spec] = (st, loop)
        snap = loop.pool.snapshot()
        root_pages = cfg.prefix_tokens // 16
        pad_pages = 1 if cfg.graphs else 0                 # the graphs' padding session
        assert len(snap["free_queue"]) == loop.pool.num_pages - root_pages - pad_pages
    st_on, loop_on = runs[True]
    st_off, _ = runs[False]
    assert st_on.spec_batches > 0 and st_off.spec_batches == 0
    assert st_on.final_lengths == st_off.final_lengths
    c = loop_on.cfg
    want = [c.prefix_tokens + c.question_tokens + c.steps * (c.decode_tokens - 1) +
            sum(c.spec_tokens + int(loop_on.tool_len[i, k]) for k in range(c.steps - 1))
            for i in range(c.sessions)]
    assert st_on.final_lengths == want
