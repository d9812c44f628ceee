"""Small, self-contained launches of each hot kernel, sized for Nsight Compute captures.

    python -m loopfuse_b200.profile_cases decode  [--sessions 32] [--reps 3]
    python -m loopfuse_b200.profile_cases prefill [--batch 2] [--seq 4096] [--reps 3]
    python -m loopfuse_b200.profile_cases pool
    python -m loopfuse_b200.profile_cases paged [--sessions 128] [--reps 3]
    python -m loopfuse_b200.profile_cases epilogue [--tokens 16384] [--reps 3]
    python -m loopfuse_b200.profile_cases dedup [--sessions 512] [--reps 3]
    python -m loopfuse_b200.profile_cases fusion_decode [--sessions 64] [--private 600] [--reps 3]
    python -m loopfuse_b200.profile_cases projections [--rows 64] [--reps 3] [--only qkv]

Each case builds its inputs, runs one warm-up launch and then ``--reps`` launches of the op,
so a capture can skip the warm-up (``-s``) and take one to three launches (``-c``).  The decode
case keeps the headline distribution (lengths U[1024, 32768], 2048-token shared prefix) with
fewer sessions: 32 sessions hold ~2.2 GB of K/V, larger than L2.
"""
from __future__ import annotations

import argparse

import torch

from . import attention as att
from .workloads import decode_bytes, decode_inputs, prefill_flops, prefill_inputs


def _event_ms(fn, reps: int) -> float:
    """CUDA-event time per call of ``reps`` back-to-back calls of ``fn`` (after one warm-up call
    by the caller); each call is one launch, so a profiler can skip the warm-up and take some."""
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(max(1, reps)):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / max(1, reps)


def run_decode(sessions: int, reps: int, pps: int) -> None:
    w = decode_inputs(N=sessions, seed=0)
    max_pages = w.block_table.shape[1]
    pps = pps or att.default_pages_per_split(sessions, w.k_pages.shape[1], max_pages, w.n_prefix_pages)
    out = torch.empty_like(w.q)
    ws = torch.empty(att.decode_workspace_bytes(sessions, w.q.shape[1], w.q.shape[2], max_pages, pps,
                                                w.n_prefix_pages), dtype=torch.uint8, device="cuda")
    for _ in range(1 + reps):
        att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                         num_prefix_pages=w.n_prefix_pages, pages_per_split=pps, out=out,
                         workspace=ws)
    torch.cuda.synchronize()
    b = decode_bytes(w)
    print(f"decode sessions={sessions} pages_per_split={pps} unique_bytes={b['unique']} "
          f"suffix_kv_bytes={b['suffix_kv']}")


def run_fusion_decode(sessions: int, reps: int, pps: int, private: int, layers: int = 4) -> None:
    """One decode call of the KV-fusion loop's shape: ``sessions`` sessions sharing a 4096-token
    prefix, each with about ``private`` tokens of its own (uniform in [private/2, 3private/2]),
    Llama-3-8B attention shapes.  ``layers`` independent pools are cycled, as the loop's layers
    are, so successive calls do not find their pages in L2.  Prints the CUDA-event time per call
    and the algorithmic bytes."""
    g = torch.Generator().manual_seed(3)
    lens = [4096 + int(x) for x in torch.randint(private // 2, 3 * private // 2 + 1, (sessions,),
                                                 generator=g)]
    ws_ = [decode_inputs(N=sessions, lengths=lens, prefix_tokens=4096, seed=l) for l in range(layers)]
    w0 = ws_[0]
    max_pages = w0.block_table.shape[1]
    pps = pps or att.default_pages_per_split(sessions, 8, max_pages, w0.n_prefix_pages)
    out = torch.empty_like(w0.q)
    ws = torch.empty(att.decode_workspace_bytes(sessions, 32, 128, max_pages, pps, w0.n_prefix_pages),
                     dtype=torch.uint8, device="cuda")

    def call(w):
        att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                         num_prefix_pages=w.n_prefix_pages, pages_per_split=pps, out=out, workspace=ws)
    for w in ws_:
        call(w)
    torch.cuda.synchronize()
    # The loop replays its decode calls from a CUDA graph; so does this case (host launch cost
    # would otherwise exceed the GPU time of a call).
    per_graph = 8 * layers
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            for i in range(per_graph):
                call(ws_[i % layers])
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(max(1, reps)):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (max(1, reps) * per_graph)
    b = decode_bytes(w0)
    print(f"fusion decode sessions={sessions} private~{private} pages_per_split={pps} "
          f"unique_bytes={b['unique']} suffix_kv_bytes={b['suffix_kv']} ms_per_call={ms:.4f} "
          f"GBps={b['unique'] / ms / 1e6:.1f}")


def run_prefill(batch: int, seq: int, reps: int) -> None:
    q, k, v = prefill_inputs(batch, 32, 8, seq, 128, seed=0)
    att.prefill_attention_fwd(q, k, v, causal=True)
    ms = _event_ms(lambda: att.prefill_attention_fwd(q, k, v, causal=True), reps)
    fl = prefill_flops(batch, 32, seq, 128)
    print(f"prefill B={batch} S={seq} flops={fl:.4e} ms_per_call={ms:.4f} TFLOPs={fl / ms / 1e9:.1f}")


def run_pool(reps: int) -> None:
    from .runtime.kv_pool import KVPool
    pool = KVPool(num_layers=32, num_heads=32, num_kv_heads=8, head_dim=128, max_seq_len=8192,
                  max_slots=65, dtype=torch.bfloat16)
    src = pool.alloc()
    kk = torch.randn(32, 4096, 8, 128, dtype=torch.bfloat16, device="cuda")
    pool.append([src], [kk], [kk])
    for _ in range(1 + reps):
        forks = pool.fork(src, 4096, n=64)
        new = [torch.randn(32, 120, 8, 128, dtype=torch.bfloat16, device="cuda") for _ in forks]
        pool.append(forks, new, new)
        pool.block_table(forks)
        pool.release_all(forks)
    torch.cuda.synchronize()
    print("pool fork/append/free x", 1 + reps)


def run_paged(sessions: int, reps: int) -> None:
    """Agent-shaped paged prefill: tool outputs (geometric, mean 120, cap 1024) appended after
    a 4096-token shared prefix, Llama-3-8B attention shapes, one layer of pages."""
    import numpy as np
    from .runtime.kv_pool import KVPool
    rng = np.random.default_rng(0)
    lens = [int(x) for x in np.minimum(rng.geometric(1 / 120, size=sessions), 1024)]
    pool = KVPool(num_layers=1, num_heads=32, num_kv_heads=8, head_dim=128, max_seq_len=8192,
                  max_slots=sessions + 1, dtype=torch.bfloat16,
                  num_pages=256 + sum((n + 15) // 16 for n in lens) + 16)
    root = pool.alloc()
    kk = torch.randn(4096, 8, 128, device="cuda").bfloat16()
    pool.write_layer([root], pool.reserve([root], [4096]), 0, kk, kk, [4096])
    ss = pool.fork(root, 4096, n=sessions)
    T = sum(lens)
    kn = torch.randn(T, 8, 128, device="cuda").bfloat16()
    pool.write_layer(ss, pool.reserve(ss, lens), 0, kn, kn, lens)
    q = torch.randn(T, 32, 128, device="cuda").bfloat16()
    table, sl = pool.block_table(ss)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    kp, vp = pool.layer_pages(0)
    att.prefill_paged(q, kp, vp, table, cu, sl, max(lens))
    ms = _event_ms(lambda: att.prefill_paged(q, kp, vp, table, cu, sl, max(lens)), reps)
    fl = sum(4 * 128 * 32 * n * 4096 + 4 * 128 * 32 * n * (n + 1) // 2 for n in lens)
    print(f"paged prefill sessions={sessions} new_tokens={T} flops={fl:.4e} ms_per_call={ms:.4f} "
          f"TFLOPs={fl / ms / 1e9:.1f}")


def run_epilogue(tokens: int, reps: int) -> None:
    """Decoder epilogues at Llama-3-8B shapes: fused QKV split + RoPE + page scatter, residual
    add + RMSNorm, SwiGLU gate."""
    from . import model_ops as mo
    from .runtime.kv_pool import KVPool
    n_sess = 16
    per = tokens // n_sess
    pool = KVPool(num_layers=1, num_heads=32, num_kv_heads=8, head_dim=128,
                  max_seq_len=per + 16, max_slots=n_sess, dtype=torch.bfloat16)
    ss = [pool.alloc() for _ in range(n_sess)]
    start = pool.reserve(ss, [per] * n_sess)
    qkv = torch.randn(per * n_sess, 48 * 128, device="cuda").bfloat16()
    q = torch.empty(per * n_sess, 32, 128, dtype=torch.bfloat16, device="cuda")
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, device="cuda").float() / 128))
    ang = torch.arange(per + 16, device="cuda").float()[:, None] * inv[None, :]
    rope = (ang.cos().contiguous(), ang.sin().contiguous())
    x = torch.randn(per * n_sess, 4096, device="cuda").bfloat16()
    d = torch.randn_like(x)
    w = torch.ones(4096, dtype=torch.bfloat16, device="cuda")
    gu = torch.randn(per * n_sess, 2 * 14336, device="cuda").bfloat16()
    for _ in range(1 + reps):
        pool.write_qkv(ss, start, 0, qkv, q, [per] * n_sess, rope=rope)
        mo.add_rmsnorm(x, d, w, 1e-5)
        mo.swiglu(gu)
    torch.cuda.synchronize()
    print(f"epilogue tokens={per * n_sess}")


def run_dedup(sessions: int, reps: int) -> None:
    """Register one 4096-token prompt, then dedup ``sessions`` requests sharing it."""
    from .runtime.kv_pool import KVPool
    pool = KVPool(num_layers=1, num_heads=8, num_kv_heads=8, head_dim=64, max_seq_len=4096,
                  max_slots=sessions + 1, dtype=torch.bfloat16, num_pages=512)
    root = pool.alloc()
    pool.reserve([root], [4096])
    prompt = torch.randint(0, 128000, (4096,), dtype=torch.int32).tolist()
    pool.register_prefix(root, prompt)
    ss = [pool.alloc() for _ in range(sessions)]
    for _ in range(1 + reps):
        pool.dedup_prefix(ss, [prompt] * sessions)
        pool.free(ss)
    torch.cuda.synchronize()
    print(f"dedup sessions={sessions} pages={4096 // 16}")


LLAMA_PROJECTIONS = {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 28672),
                     "down": (14336, 4096), "lm_head": (4096, 128256)}


def run_projections(rows: int, reps: int, only: str = "") -> None:
    """The decoder's dense projections (Llama-3-8B shapes) at a decode batch of ``rows`` rows:
    ``lf_gemm_skinny`` against the library GEMM (``torch.matmul``), both replayed from CUDA
    graphs over enough weight copies (>= 4, >= 512 MB) that no launch finds its weights in L2.
    Prints the CUDA-event time per call, the weight bytes per call and the max difference of the
    two results.  Under a profiler the graphs still replay, one kernel launch per call."""
    from . import model_ops as mo
    names = [only] if only else list(LLAMA_PROJECTIONS)
    g = torch.Generator(device="cuda").manual_seed(0)
    for name in names:
        k, n = LLAMA_PROJECTIONS[name]
        copies = max(4, -(-(512 << 20) // (k * n * 2)))
        ws = [(torch.randn(k, n, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
              for _ in range(copies)]
        x = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
        y0 = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
        y1 = torch.empty_like(y0)
        wsp = torch.empty(mo.skinny_workspace_bytes(rows, n, k, torch.cuda.get_device_properties(0)
                                                    .multi_processor_count),
                          dtype=torch.uint8, device="cuda")
        calls = {"skinny": lambda w: mo.gemm_skinny(x, w, out=y0, workspace=wsp),
                 "library": lambda w: torch.matmul(x, w, out=y1)}
        res = {}
        for tag, fn in calls.items():
            for w in ws:
                fn(w)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                with torch.cuda.graph(graph):
                    for w in ws:
                        fn(w)
            torch.cuda.current_stream().wait_stream(side)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(max(1, reps)):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            res[tag] = e0.elapsed_time(e1) * 1e3 / (max(1, reps) * copies)
        fn = calls["skinny"]
        fn(ws[-1])
        torch.matmul(x, ws[-1], out=y1)
        torch.cuda.synchronize()
        diff = (y0.float() - y1.float()).abs().max().item()
        wb = k * n * 2
        print(f"projection {name} M={rows} K={k} N={n} weight_bytes={wb} "
              f"skinny_us={res['skinny']:.2f} ({wb / res['skinny'] / 1e3:.0f} GB/s) "
              f"library_us={res['library']:.2f} ({wb / res['library'] / 1e3:.0f} GB/s) "
              f"max_diff={diff:.3e}", flush=True)
        del ws


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["decode", "prefill", "pool", "paged", "epilogue", "dedup",
                                     "fusion_decode", "projections"])
    ap.add_argument("--only", default="")
    ap.add_argument("--rows", type=int, default=64)
    ap.add_argument("--private", type=int, default=600)
    ap.add_argument("--sessions", type=int, default=32)
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--pages-per-split", type=int, default=0)
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    if a.case == "decode":
        run_decode(a.sessions, a.reps, a.pages_per_split)
    elif a.case == "fusion_decode":
        run_fusion_decode(a.sessions, a.reps, a.pages_per_split, a.private)
    elif a.case == "projections":
        run_projections(a.rows, a.reps, a.only)
    elif a.case == "prefill":
        run_prefill(a.batch, a.seq, a.reps)
    elif a.case == "paged":
        run_paged(a.sessions, a.reps)
    elif a.case == "epilogue":
        run_epilogue(a.tokens, a.reps)
    elif a.case == "dedup":
        run_dedup(a.sessions, a.reps)
    else:
        run_pool(a.reps)


if __name__ == "__main__":
    main()
