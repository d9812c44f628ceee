"""GPT-2-small 3-step ReAct program: GPU path (sm_100a attention + device pool) vs the CPU
program (fp32 SDPA, pool oracle), teacher-forced on the CPU program's tokens.

The GPU model keeps the dense math in fp32 and runs attention in bf16, so the comparison is
the attention tolerance: per chunk and layer, the attention output at the chunk's last
position within max-abs 2e-2 and mean-abs 2e-3 of the fp32 program (the values are O(0.1)).
Block tables after each step and the sequence lengths must be identical (page reuse included:
the forked prefix pages are shared, the tool / decode pages come from the FIFO queue in the
same order).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def programs():
    from oracle.gpt2_program import GPT2Program, gpt2_weights
    from loopfuse_b200.gpt2 import GPT2Config, GPT2Model, run_react

    torch.backends.cuda.matmul.allow_tf32 = False
    prog = GPT2Program()
    ref = prog.run()
    chunks, toks, off = {}, ref.tokens, 0
    parts = []
    for kind, start, n in ref.chunks:
        parts.append((kind, toks[off:off + n]))
        off += n
    prefix = [p for k, p in parts if k == "prefix"][0]
    prompts = [p for k, p in parts if k == "prompt"]
    tools = [p for k, p in parts if k == "tool"]
    model = GPT2Model(GPT2Config(), weights=gpt2_weights(prog.cfg, 0), device="cuda")
    got = run_react(model, prefix, prompts, tools, decode_tokens=prog.DECODE,
                    forced=ref.choices, record=True,
                    num_pages=prog.pool.num_pages)
    return ref, got


def test_program_shape(programs):
    ref, got = programs
    assert ref.lengths == [822, 1062, 1222]
    assert got.lengths == ref.lengths
    assert len(got.attn_last) == len(ref.attn_last) == len(ref.chunks)


def test_block_tables_bit_exact(programs):
    ref, got = programs
    for step, (a, b) in enumerate(zip(got.tables, ref.tables)):
        assert a == b, f"block table differs after step {step}"


def test_attention_outputs_within_tolerance(programs):
    ref, got = programs
    worst_max = worst_mean = 0.0
    for i, (a, b) in enumerate(zip(got.attn_last, ref.attn_last)):
        d = (a - b).abs()
        worst_max = max(worst_max, d.max().item())
        worst_mean = max(worst_mean, d.mean().item())
        assert d.max().item() <= 2e-2, f"chunk {i} {ref.chunks[i]}: max-abs {d.max().item():.3e}"
        assert d.mean().item() <= 2e-3, f"chunk {i} {ref.chunks[i]}: mean-abs {d.mean().item():.3e}"
    print(f"gpt2 program: worst max-abs {worst_max:.3e}, worst mean-abs {worst_mean:.3e}")


def test_greedy_choices_mostly_agree(programs):
    """Random-weight logits have near ties; bf16 attention may flip a few of them."""
    ref, got = programs
    agree = sum(a == b for a, b in zip(got.choices, ref.choices)) / len(ref.choices)
    assert agree >= 0.8, f"only {agree:.0%} of greedy choices agree"
