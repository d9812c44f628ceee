"""Speculative prefill through the executor: a hit adopts the speculative branch, a miss frees it.

The program is a 2-step GPT-2 ReAct program (head_dim 64 attention on the sm_100a kernels, fp32
dense math, device pool) run through ``SpecPrefillPass`` + ``PhaseSelectPass``: step 0 prefills
the prompt and calls a 120 ms tool, in front of which the pass puts a speculative prefill;
step 1 prefills the observation and decodes.  The model predicts the observation tokens
(``spec_tokens``): equal to the real ones (hit) or not (miss).  Either way the decoded tokens
must equal those of a run without speculation, and the pool metadata -- after the speculative
prefill, after the decode and after the run -- must equal the pool oracle's replay of the same
operations bit for bit (reference ``runtime/executor.py:238-249``, ``passes/spec_prefill.py``).
"""
import pytest
import torch

from oracle.pool_spec import PagedKVPoolSpec
from loopfuse_b200.gpt2 import GPT2Config, GPT2Model
from loopfuse_b200.ir.builder import AgentProgramBuilder
from loopfuse_b200.ir.dialect import GPT2_CONFIG, GPT2_KV_CONFIG, KernelTarget, LLMForwardOp, Phase
from loopfuse_b200.passes import PassManager, PhaseSelectPass, SpecPrefillPass
from loopfuse_b200.runtime.executor import AgentExecutor

pytestmark = pytest.mark.gpu

SYS, Q, OBS, DEC = 200, 37, 29, 5          # 237-token prompt: the fork copies a partial page
PAGES, SLOTS = 64, 3


class SpecModel:
    """GPT-2 plus the tokens of one request and a prediction of the step-1 observation."""

    def __init__(self, model, prompt, obs, predicted=None):
        self.m, self.prompt, self.obs = model, prompt, obs
        if predicted is not None:
            self.spec_tokens = lambda step_id: predicted

    def prompt_tokens(self, step_id, seq_len):
        return self.prompt if step_id == 0 else self.obs

    def prefill(self, tokens, kv_state, attention=None):
        return self.m.prefill(tokens, kv_state, attention)

    def decode(self, tokens, kv_state, attention=None):
        return self.m.decode(tokens, kv_state, attention)


def _program(speculate: bool):
    cfg = dict(GPT2_CONFIG, system_prompt_len=SYS)
    b = AgentProgramBuilder("spec", cfg, GPT2_KV_CONFIG)
    b.add_react_step(0, "search", 120.0, is_first_step=True, system_prompt_len=SYS + Q)
    b.add_react_step(1, "lookup", 1.0)                    # too short a window to speculate
    prog = b.set_target(KernelTarget.CUDA).build()
    step1 = prog.steps[1]
    dec = step1.llm_ops()[0]
    step1.insert_before(dec, LLMForwardOp(dec.operands[0], prog.kv_state, cfg,
                                          phase=Phase.PREFILL, seq_len=OBS))
    passes = ([SpecPrefillPass()] if speculate else []) + [PhaseSelectPass(hardware="b200")]
    PassManager(passes).run(prog)
    return prog


@pytest.fixture(scope="module")
def model():
    torch.backends.cuda.matmul.allow_tf32 = False
    return GPT2Model(GPT2Config(), seed=5)


@pytest.fixture(scope="module")
def tokens():
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, 50257, (SYS + Q,), generator=g).cuda()
    obs = torch.randint(0, 50257, (OBS,), generator=g).cuda()
    return prompt, obs


def _run(model, prompt, obs, predicted, speculate):
    pool = model.new_pool(num_pages=PAGES, max_slots=SLOTS)
    snaps = []

    def tool(_):
        torch.cuda.synchronize()
        snaps.append(pool.snapshot())
        return "ok"
    exe = AgentExecutor(SpecModel(model, prompt, obs, predicted), pool,
                        tools={"search": tool, "lookup": tool}, max_decode_tokens=DEC)
    res = exe.run(_program(speculate), "q")
    torch.cuda.synchronize()
    return res, snaps, pool


def _same(snap, spec):
    want = spec.snapshot()
    assert snap["status"] == 0
    for key in ("free_queue", "refcount", "block_table", "seq_len"):
        assert snap[key] == want[key], key


def test_program_gets_one_speculative_prefill():
    prog = _program(True)
    kinds = [type(o).__name__ for o in prog.steps[0].act_region]
    assert kinds == ["ParseActionOp", "SpeculativePrefillOp", "ToolCallOp"]
    assert not any(type(o).__name__ == "SpeculativePrefillOp" for o in prog.steps[1].all_ops())


@pytest.mark.parametrize("hit", [True, False])
def test_speculation_matches_the_plain_run_and_the_pool_spec(model, tokens, hit):
    prompt, obs = tokens
    predicted = obs.clone() if hit else torch.roll(obs, 1)
    plain, _, _ = _run(model, prompt, obs, None, speculate=False)
    got, snaps, pool = _run(model, prompt, obs, predicted, speculate=True)

    assert got.step_traces[1].spec_prefill_hit is hit
    assert plain.step_traces[1].spec_prefill_hit is False
    assert got.step_traces[1].output_tokens == plain.step_traces[1].output_tokens
    assert len(got.step_traces[1].output_tokens) == DEC

    spec = PagedKVPoolSpec(PAGES, SLOTS, pool.max_pages_per_seq)
    a = spec.open_seq()
    spec.reserve([a], [SYS + Q])
    b = spec.open_seq()                          # the speculative branch
    spec.fork(a, [b], SYS + Q)
    spec.reserve([b], [OBS])
    _same(snaps[0], spec)                        # during step 0's tool call
    if hit:                                      # adopt: a's pages dropped, its row recycled
        spec.free([a])
        spec.free_seqs.append(a)
        live = b
    else:                                        # miss: the branch is released
        spec.close_seq(b)
        spec.reserve([a], [OBS])
        live = a
    for _ in range(DEC):
        spec.reserve([live], [1])
    _same(snaps[1], spec)                        # during step 1's tool call
    spec.close_seq(live)
    _same(pool.snapshot(), spec)                 # after the run
    assert pool._free_slots == spec.free_seqs
