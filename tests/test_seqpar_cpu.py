"""Sequence-parallel bidirectional scan: the carry exchange and fold, run as
world_size 2 and 3 gloo process groups on CPU with the f64 oracle standing in
for the GPU scan.  Each rank's segment of the merged output must equal the
same slice of the unsplit bidirectional scan."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _oracle_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                 return_last_state=False, initial_state=None, reverse=False):
    import oracle
    n = lambda t: None if t is None else t.numpy()  # noqa: E731
    out, last = oracle.m1_scan(n(u), n(delta), n(A), n(B), n(C), D=n(D), z=n(z),
                               delta_bias=n(delta_bias), delta_softplus=delta_softplus,
                               reverse=reverse, h0=n(initial_state))
    out, last = torch.from_numpy(out), torch.from_numpy(last)
    return (out, last) if return_last_state else out


def _oracle_state(u, delta, A, B, C, delta_bias=None, delta_softplus=False, reverse=False,
                  initial_state=None):
    return _oracle_scan(u, delta, A, B, C, delta_bias=delta_bias, delta_softplus=delta_softplus,
                        reverse=reverse, initial_state=initial_state, return_last_state=True)[1]


def _case(L):
    rng = np.random.default_rng(0)
    Bsz, Dd, N = 2, 5, 16
    f = lambda *s: torch.from_numpy(rng.standard_normal(s))  # noqa: E731
    return dict(u=f(Bsz, Dd, L), delta=0.5 * f(Bsz, Dd, L),
                A=-torch.from_numpy(np.exp(rng.uniform(np.log(0.5), np.log(16), (Dd, N)))),
                B=f(Bsz, N, L), C=f(Bsz, N, L), D=f(Dd), z=f(Bsz, Dd, L),
                delta_bias=torch.from_numpy(rng.uniform(-6, -3, Dd)), delta_softplus=True)


def _worker(rank, world, port, L, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "oracle")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from armhackathon_b200.seqpar import bidirectional_scan_seqpar
    x = _case(L)
    cuts = np.linspace(0, L, world + 1).astype(int)
    sl = slice(cuts[rank], cuts[rank + 1])
    tv = ("u", "delta", "B", "C", "z")
    mine = {k: (v[..., sl].contiguous() if k in tv else v) for k, v in x.items()}
    got = bidirectional_scan_seqpar(**mine, scan_fn=_oracle_scan, state_fn=_oracle_state)
    full = _oracle_scan(**x) + _oracle_scan(**x, reverse=True)
    err = float((got - full[..., sl]).abs().max() / full.abs().max())
    q.put((rank, err))
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world,L", [(2, 300), (3, 257)])
def test_seqpar_bidirectional_matches_unsplit(world, L):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, L, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    errs = dict(q.get(timeout=10) for _ in range(world))
    assert max(errs.values()) < 1e-8, errs  # f64: exp(A*sum dt) vs prod exp(A*dt)


def test_fold_carries_single_process():
    from armhackathon_b200.seqpar import fold_carries
    A = -torch.rand(3, 4, dtype=torch.float64)
    h = [torch.rand(1, 3, 4, dtype=torch.float64) for _ in range(3)]
    s = [torch.rand(1, 3, dtype=torch.float64) for _ in range(3)]
    d = [torch.exp(A[None] * si[..., None]) for si in s]
    assert torch.allclose(fold_carries(h, s, A, 2, False), d[1] * h[0] + h[1])
    assert torch.allclose(fold_carries(h, s, A, 0, True), d[1] * h[2] + h[1])
    assert torch.equal(fold_carries(h, s, A, 0, False), torch.zeros_like(h[0]))
