"""Small, self-contained launches of each hot kernel, sized for Nsight Compute captures.

    python -m loopfuse_b200.profile_cases decode  [--sessions 32] [--reps 3]
    python -m loopfuse_b200.profile_cases prefill [--batch 2] [--seq 4096] [--reps 3]
    python -m loopfuse_b200.profile_cases pool

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


def run_decode(sessions: int, reps: int, pps: int) -> None:
    w = decode_inputs(N=sessions, seed=0)
    max_pages = w.block_table.shape[1]
    pps = pps or att.default_pages_per_split(sessions, w.k_pages.shape[1], max_pages)
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


def run_prefill(batch: int, seq: int, reps: int) -> None:
    q, k, v = prefill_inputs(batch, 32, 8, seq, 128, seed=0)
    for _ in range(1 + reps):
        att.prefill_attention_fwd(q, k, v, causal=True)
    torch.cuda.synchronize()
    print(f"prefill B={batch} S={seq} flops={prefill_flops(batch, 32, seq, 128):.4e}")


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


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["decode", "prefill", "pool"])
    ap.add_argument("--sessions", type=int, default=32)
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--pages-per-split", type=int, default=0)
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    if a.case == "decode":
        run_decode(a.sessions, a.reps, a.pages_per_split)
    elif a.case == "prefill":
        run_prefill(a.batch, a.seq, a.reps)
    else:
        run_pool(a.reps)


if __name__ == "__main__":
    main()
