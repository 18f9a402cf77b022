"""The give-up path of the tensor-core kernels, on real calls (a B200 with -m gpu).

Every mbarrier wait in the kernels is bounded; a wait that gives up records a code in the
device status word and sets the abort flag of every CTA of its cluster, every role unwinds,
and each CTA lets the asynchronous copies, stores and MMAs already aimed at it land before
it releases its shared and tensor memory.  Here the bound is set to 1 us (option 3), far
below the pipeline's own latencies, so the waits give up mid-pipeline on real calls: the
persistent four-CTA pair kernel at a C3-like shape, the pair kernel in split mode with
the combine kernel (C1), and the two-CTA kernel.  (The bf16 multi-head kernel's waits end
within the polls that precede each time check, so a short bound does not make them give
up; its path is read-checked only.)  The call
must report a timeout in the device status (not lose the context), and the same call
with the normal bound must then be correct.  Each case runs in a child process, so this
file cannot disturb the other tests whatever happens.
"""

import multiprocessing as mp

import pytest

import mp_workers

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["pair", "split", "two_cta"])
def test_give_up_then_normal_call(kind):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    proc = ctx.Process(target=mp_workers.give_up_worker, args=(kind, results))
    proc.start()
    try:
        st1, err, st2, exc = results.get(timeout=300)
    finally:
        proc.join(timeout=60)
        if proc.is_alive():
            proc.kill()
    assert exc is None, exc
    assert st1 is not None and st1 > 0, f"{kind}: no timeout reported (status {st1})"
    assert st2 == 0, f"{kind}: status {st2} after the normal call"
    assert err <= 2e-3, f"{kind}: {err:.2e} after the give-up"
