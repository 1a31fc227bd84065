"""praxis_b200_dispatch_noalloc (scratch in a static device array) against
praxis_b200_dispatch (caller workspace): the same outputs, bit for bit, on
calls in a row with different inputs, so a call that read scratch left by
the previous one would show. Collected last on purpose: it must pass after
every other test has used the library in the same process, and alone."""

from __future__ import annotations

import pytest
import torch
from conftest import assert_bytes_equal, pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    p = pkg()
    p.capi.load()
    return p


def _inputs(t, e, k, seed, concentrated=False):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(t, e, generator=g)
    if concentrated:
        logits[: (3 * t) // 4, 0] += 50.0
    top = logits.topk(k, -1).indices.contiguous()
    gate = torch.softmax(torch.randn(t, k, generator=g), -1).to(torch.bfloat16)
    x = torch.randn(t, 256, generator=g).to(torch.bfloat16)
    return top.to(DEV), gate.to(DEV), x.to(DEV)


def _outputs(P, t, e, k):
    r = t * k
    max_tiles = max(P.ops.padded_rows(r, e) // 128, 1)
    i64 = dict(dtype=torch.int64, device=DEV)
    i32 = dict(dtype=torch.int32, device=DEV)
    # sentinel fill: a stale or missing write shows as a mismatch
    return dict(
        order=torch.full((r,), -7, **i64), inverse=torch.full((r,), -7, **i64), tokens=torch.full((r,), -7, **i64),
        tokens32=torch.full((r,), -7, **i32), sorted_gate=torch.full((r,), -7.0, dtype=torch.bfloat16, device=DEV),
        offsets=torch.full((e,), -7, **i32), csr=torch.full((e + 1,), -7, **i32),
        pcsr=torch.full((e + 1,), -7, **i32), tiles=torch.full((2 * max_tiles, 4), -7, **i32),
        num_tiles=torch.full((2,), -7, **i32), act_global=torch.full((e,), -7.0, dtype=torch.float32, device=DEV),
        act_amax=torch.full((e,), -7, **i32))


def _compare(P, got, want, e):
    n_tiles, n_pairs = (int(v) for v in want.num_tiles.cpu())
    max_tiles = got["tiles"].shape[0] // 2
    assert [int(v) for v in got["num_tiles"].cpu()] == [n_tiles, n_pairs]
    assert_bytes_equal(got["tiles"][:n_tiles].cpu(), want.tiles[:n_tiles].cpu())
    assert_bytes_equal(got["tiles"][max_tiles:max_tiles + n_pairs].cpu(),
                       want.tiles[max_tiles:max_tiles + n_pairs].cpu())
    for name, ref in [("order", want.order), ("inverse", want.inverse), ("tokens", want.tokens),
                      ("tokens32", want.tokens32), ("sorted_gate", want.sorted_gate), ("offsets", want.offsets),
                      ("csr", want.csr), ("pcsr", want.pcsr), ("act_global", want.act_global),
                      ("act_amax", want.act_amax)]:
        assert_bytes_equal(got[name].cpu(), ref.cpu())


# Calls in a row, alternating sizes: later calls reuse the scratch that
# earlier calls wrote with other counts.
SEQUENCE = [(4096, 64, 4, False), (333, 8, 2, False), (16384, 256, 8, True), (1, 8, 1, False),
            (2048, 128, 8, False), (700, 16, 2, True)]


def test_dispatch_noalloc_matches_dispatch_on_calls_in_a_row(P):
    for i, (t, e, k, conc) in enumerate(SEQUENCE):
        top, gate, x = _inputs(t, e, k, seed=100 + i, concentrated=conc)
        amax = P.ops.row_amax(x)
        want = P.ops.dispatch(top, gate, e, amax)
        got = _outputs(P, t, e, k)
        P.ops.dispatch_noalloc(top, gate, e, amax, **got)
        torch.cuda.synchronize()
        _compare(P, got, want, e)
    assert P.capi.device_error(torch.cuda.current_device()) == 0


def test_dispatch_noalloc_twice_on_the_same_input(P):
    top, gate, x = _inputs(3000, 32, 2, seed=7)
    amax = P.ops.row_amax(x)
    want = P.ops.dispatch(top, gate, 32, amax)
    for _ in range(2):
        got = _outputs(P, 3000, 32, 2)
        P.ops.dispatch_noalloc(top, gate, 32, amax, **got)
        torch.cuda.synchronize()
        _compare(P, got, want, 32)


def test_dispatch_noalloc_rejects_sizes_beyond_its_scratch(P):
    t, e, k = 140_000, 1024, 1  # needs ~4.5 MB of scratch: over the static 4 MiB + 256
    lib = P.capi.load()
    assert lib.praxis_b200_dispatch_workspace_size(t, k, e) > (4 << 20) + 256
    top = torch.zeros(t, k, dtype=torch.int64, device=DEV)
    gate = torch.ones(t, k, dtype=torch.bfloat16, device=DEV)
    got = _outputs(P, t, e, k)
    with pytest.raises(ValueError, match="static scratch"):
        P.ops.dispatch_noalloc(top, gate, e, None, **got)
    # nothing was launched: the outputs keep their sentinel
    assert int(got["num_tiles"][0].item()) == -7
