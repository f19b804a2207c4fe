"""The C ABI is reentrant: calls from several host threads, each on its own
CUDA stream, run side by side and give what the same calls give one after
another (the kernels are deterministic, so bit for bit).  XLA may call a
custom-call handler from several threads on different streams; ctypes releases
the GIL for the duration of each call, so the host sides really overlap."""

import threading

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, B=1, T=512, H=4):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=gen, device="cuda")  # noqa: E731
    q = torch.nn.functional.normalize(rn(B, T, H, 128), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(rn(B, T, H, 128), dim=-1).to(torch.bfloat16)
    v = rn(B, T, H, 128).to(torch.bfloat16)
    g = torch.nn.functional.logsigmoid(rn(B, T, H, 128) + 3.0).to(torch.bfloat16)
    beta = torch.sigmoid(rn(B, T, H)).to(torch.bfloat16)
    do = rn(B, T, H, 128).to(torch.bfloat16)
    return q, k, v, g, beta, do


def _step(x):
    from axiom_b200 import kda_bwd, kda_fwd

    q, k, v, g, beta, do = x
    o, s_t, ck = kda_fwd(q, k, v, g, beta, None, chunk=64, need_ckpt=True)
    grads = kda_bwd(q, k, v, g, beta, ck, do, None, chunk=64, need_ds0=False)
    return [o, s_t] + list(grads[:5])


def test_threads_on_their_own_streams_match_sequential_calls():
    n_threads, n_iter = 4, 6
    xs = [_inputs(100 + i) for i in range(n_threads)]
    torch.cuda.synchronize()
    ref = [_step(x) for x in xs]
    torch.cuda.synchronize()
    got, errors = [None] * n_threads, []
    start = threading.Barrier(n_threads)

    def worker(i):
        try:
            s = torch.cuda.Stream()
            start.wait()
            with torch.cuda.stream(s):
                for _ in range(n_iter):
                    out = _step(xs[i])
            s.synchronize()
            got[i] = out
        except Exception as e:  # reported below, on the main thread
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(n_threads)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for i in range(n_threads):
        for a, b in zip(got[i], ref[i]):
            assert torch.equal(a, b), i
