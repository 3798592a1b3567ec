"""Bounded device-side waits run to expiry on one GPU.

The cross-rank flag wait of the sharded update (``rf_flags_wait``) polls with
a ``%globaltimer`` limit; when the limit passes it sets the peer error word
and lets the stream move on instead of hanging.  Here the wait is given a
flag array in this GPU's own memory that nothing ever signals and a 50 ms
limit, so it gives up by design: no fault, no hang, and the context stays
usable.  The test checks the non-blocking snapshot of the error words, the
RF_ETIMEOUT report of ``rf_sync_check`` (which clears the word), and the
sharded update's ``ErrorWatch`` raising on such a snapshot.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from rollfast_b200 import _lib as L

    L.load()
    return L


def test_flag_wait_gives_up_and_reports_timeout(cuda_device):
    L = _lib()
    stream = torch.cuda.current_stream(cuda_device)
    flags = torch.zeros(4, dtype=torch.int32, device=cuda_device)  # never signalled
    snap = torch.full((2,), -1, dtype=torch.int32, pin_memory=True)
    L.sync_check(stream.cuda_stream)  # start from clear error words
    L.flags_wait(flags.data_ptr(), 4, -1, 1, 0.05, stream.cuda_stream)
    L.error_snapshot(snap.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    assert snap.tolist() == [0, 1]  # tensor-core word clear, peer word set
    with pytest.raises(L.RollfastError) as info:
        L.sync_check(stream.cuda_stream)
    assert info.value.status == L.RF_ETIMEOUT
    L.sync_check(stream.cuda_stream)  # the report cleared the word
    L.error_snapshot(snap.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    assert snap.tolist() == [0, 0]
    x = torch.arange(8, dtype=torch.float32, device=cuda_device)
    assert float(x.sum()) == 28.0  # the context is still usable


def test_flag_wait_returns_once_signalled(cuda_device):
    L = _lib()
    stream = torch.cuda.current_stream(cuda_device)
    flags = torch.zeros(3, dtype=torch.int32, device=cuda_device)
    L.sync_check(stream.cuda_stream)
    base = flags.data_ptr()
    L.flags_signal([base + 4 * i for i in range(3)], 7, stream.cuda_stream)
    L.flags_wait(base, 3, 1, 7, 5.0, stream.cuda_stream)  # all reached (slot 1 skipped)
    L.sync_check(stream.cuda_stream)
    assert flags.tolist() == [7, 7, 7]


def test_error_watch_raises_on_a_step_whose_wait_gave_up(cuda_device):
    from rollfast_b200.distributed import ErrorWatch

    L = _lib()
    stream = torch.cuda.current_stream(cuda_device)
    L.sync_check(stream.cuda_stream)
    watch = ErrorWatch()
    watch.snapshot(stream, 1)
    watch.check(block=True)  # step 1 clean
    flags = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    L.flags_wait(flags.data_ptr(), 1, -1, 1, 0.05, stream.cuda_stream)
    watch.snapshot(stream, 2)
    with pytest.raises(L.RollfastError) as info:
        watch.check(block=True)
    assert info.value.status == L.RF_ETIMEOUT and "step 2" in str(info.value)
    L.sync_check(stream.cuda_stream)  # cleared by the report
