"""Host logic of the C-ABI communicator (g4a_dist_*), without a GPU.

g4a_dist_poll_selftest runs the deadline loop that every NCCL call of the library goes through
(non-blocking communicator: poll ncclCommGetAsyncError until the operation leaves ncclInProgress)
against the library's fake NCCL: an operation that completes, a rank that never joins (the
deadline aborts the communicator: G4A_ETIMEOUT) and a peer that fails (abort: G4A_ENCCL).  This
mirrors the reference turning a lost device into an error at the next call
(src/engine.ts:432-435, 2214, 2509).  The failure is made on the host, by the fake."""
import time

import g4attn
from g4attn._lib import STATUS_NAMES


def test_completing_operation_is_ok():
    st, aborted = g4attn.dist_poll_selftest(0, 2000)
    assert STATUS_NAMES[st] == "G4A_OK" and aborted == 0


def test_rank_that_never_joins_times_out_and_aborts():
    t0 = time.perf_counter()
    st, aborted = g4attn.dist_poll_selftest(1, 300)
    dt = time.perf_counter() - t0
    assert STATUS_NAMES[st] == "G4A_ETIMEOUT" and aborted == 1
    assert 0.25 <= dt < 5.0, dt
    msg = g4attn.load().g4a_last_error().decode()
    assert "did not join" in msg and "aborted" in msg


def test_failing_peer_aborts_with_nccl_error():
    st, aborted = g4attn.dist_poll_selftest(2, 5000)
    assert STATUS_NAMES[st] == "G4A_ENCCL" and aborted == 1
    assert "aborted" in g4attn.load().g4a_last_error().decode()
