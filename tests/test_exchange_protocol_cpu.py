"""Host restatement of the peer-memory exchange protocol of the partitioned
calls (hephaestus_b200/csrc/dist.cu, exchange_pairs_kernel), run by threads
that stand in for ranks at random speeds: every rank stores its value for call
e into entry [e % 2][rank] of every rank's mailbox, then that entry's flag = e;
then waits until every entry [e % 2][r] of its own mailbox has flag e and
reads the values.  Each value read must be the one its writer published for
call e, although fast ranks run ahead: a rank can reach call e + 2 (the same
parity) only after every rank has published call e + 1, i.e. after every rank
has finished reading call e.  The stores and flag stores are ordered like the
kernel's release store after its data stores (a lock stands in for that
ordering here); the test checks the epoch/parity argument, not the GPU's
memory model."""
import random
import threading
import time

import pytest


@pytest.mark.parametrize("nranks,calls", [(2, 300), (4, 200), (8, 100)])
def test_mailbox_protocol_under_skew(nranks, calls):
    boxes = [[[(None, 0) for _ in range(nranks)] for _ in range(2)] for _ in range(nranks)]
    lock = threading.Lock()
    errors = []

    def rank_main(rank):
        rng = random.Random(rank)
        for e in range(1, calls + 1):
            if rng.random() < 0.3:
                time.sleep(rng.random() * 1e-4)
            for r in range(nranks):  # publish: data, then the flag (one store here)
                with lock:
                    boxes[r][e & 1][rank] = ((rank, e), e)
            deadline = time.monotonic() + 20
            for r in range(nranks):  # wait for every rank's entry of this call
                while True:
                    with lock:
                        val, flag = boxes[rank][e & 1][r]
                    if flag == e:
                        break
                    if time.monotonic() > deadline:
                        errors.append(f"rank {rank} timed out on rank {r} at call {e}")
                        return
                    time.sleep(0)
                if val != (r, e):
                    errors.append(f"rank {rank} read {val} for rank {r} at call {e}")
                    return

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(nranks)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors[:3]
