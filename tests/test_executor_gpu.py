"""AgentExecutor end to end on the GPU: a built GPT-2 ReAct program, annotated by
KVFusionPass + PhaseSelectPass, runs through the sm_100a kernels (head_dim 64) and the device
pool; a second run with the same system prompt takes its pages from the prefix registry."""
import pytest
import torch

from loopfuse_b200.gpt2 import GPT2Config, GPT2Model
from loopfuse_b200.ir.builder import AgentProgramBuilder
from loopfuse_b200.ir.dialect import GPT2_CONFIG, GPT2_KV_CONFIG, KernelTarget
from loopfuse_b200.passes import KVFusionPass, PassManager, PhaseSelectPass
from loopfuse_b200.runtime.executor import AgentExecutor

pytestmark = pytest.mark.gpu

SYS_LEN, Q_LEN = 256, 40


class PromptedGPT2:
    """GPT-2 plus the prompt tokens of one request: system prompt, then a question."""

    def __init__(self, model, system, question):
        self.m, self.prompt = model, torch.tensor(system + question, dtype=torch.long, device="cuda")

    def prompt_tokens(self, step_id, seq_len):
        return self.prompt

    def prefill(self, tokens, kv_state, attention=None):
        return self.m.prefill(tokens, kv_state, attention)

    def decode(self, tokens, kv_state, attention=None):
        return self.m.decode(tokens, kv_state, attention)


def _program():
    cfg = dict(GPT2_CONFIG, system_prompt_len=SYS_LEN)
    b = AgentProgramBuilder("gpt2_react", cfg, GPT2_KV_CONFIG)
    b.add_react_step(0, "search", 1.0, is_first_step=True, system_prompt_len=SYS_LEN)
    b.add_react_step(1, "lookup", 1.0)
    b.add_react_step(2, None)
    prog = b.set_target(KernelTarget.CUDA).build()
    PassManager([KVFusionPass(), PhaseSelectPass(hardware="b200")]).run(prog)
    return prog


@pytest.fixture(scope="module")
def model():
    return GPT2Model(GPT2Config(), seed=3)


def _run(model, pool, system, question, cache=True):
    exe = AgentExecutor(PromptedGPT2(model, system, question), pool,
                        tools={"search": lambda s: "ok", "lookup": lambda s: "ok"},
                        max_decode_tokens=6, prefix_cache=cache)
    return exe.run(_program(), "question")


def test_executor_runs_and_reuses_system_prompt_pages(model):
    g = torch.Generator().manual_seed(0)
    system = torch.randint(0, 50257, (SYS_LEN,), generator=g).tolist()
    qa = torch.randint(0, 50257, (Q_LEN,), generator=g).tolist()
    qb = torch.randint(0, 50257, (Q_LEN,), generator=g).tolist()
    pool = model.new_pool(num_pages=256, max_slots=4)
    r1 = _run(model, pool, system, qa)
    t1 = r1.step_traces[0]
    assert t1.prefix_hit_tokens == 0 and t1.prefill_tokens == SYS_LEN + Q_LEN
    assert sum(len(t.output_tokens) for t in r1.step_traces) == 12      # two decode steps x 6
    r2 = _run(model, pool, system, qb)
    t2 = r2.step_traces[0]
    assert t2.prefix_hit_tokens == SYS_LEN and t2.prefill_tokens == Q_LEN
    # the same request on a fresh pool without the registry computes the same tokens
    fresh = model.new_pool(num_pages=256, max_slots=4)
    r3 = _run(model, fresh, system, qb, cache=False)
    assert [t.output_tokens for t in r3.step_traces] == [t.output_tokens for t in r2.step_traces]
    assert r3.step_traces[0].prefix_hit_tokens == 0
    # sessions are released after each run; dropping the registry frees every page
    pool.unregister_all()
    assert sorted(pool.snapshot()["free_queue"]) == list(range(pool.num_pages))


def test_non_cuda_target_raises(model):
    pool = model.new_pool(num_pages=64, max_slots=2)
    prog = _program()
    exe = AgentExecutor(PromptedGPT2(model, [1] * 16, [2] * 4), pool, tools={},
                        target=KernelTarget.TRITON, max_decode_tokens=2)
    with pytest.raises(NotImplementedError):
        exe.run(prog, "q")
