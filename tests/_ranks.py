"""Helpers for tests that run ranks as child processes."""
import queue
import time


def collect(q, procs, n, timeout):
    """n results from q; raises as soon as a rank process exits non-zero (a crashed or failed
    rank never puts its result) or when `timeout` seconds pass."""
    out = []
    deadline = time.monotonic() + timeout
    while len(out) < n:
        try:
            out.append(q.get(timeout=1.0))
            continue
        except queue.Empty:
            pass
        dead = [p for p in procs if p.exitcode not in (None, 0)]
        if dead:
            for p in procs:
                if p.is_alive():
                    p.terminate()
            raise AssertionError("rank process exited with code %s" % [p.exitcode for p in dead])
        if time.monotonic() > deadline:
            for p in procs:
                if p.is_alive():
                    p.terminate()
            raise AssertionError("ranks gave %d of %d results within %d s" % (len(out), n, timeout))
    return out
