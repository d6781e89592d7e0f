"""The landed-vector accounting of the overlapped fetch launch
(csrc/moe.cu overlap_fetch), restated step for step on the CPU: every job's
W13/S13 count must reach exactly its vector total (a job that fell short would
leave its gate/up units waiting until the bounded wait gives up), and a CTA
must publish a job only after its last chunk of that job.

The restatement mirrors the kernel's per-CTA loop (chunk base, the jobs a
chunk overlaps, the flush when the CTA's next chunk lies past the job)."""
import random

import pytest

K_CHUNK = 256 * 4   # kFetchThreads * kFetchUnroll vectors


def simulate(nm: int, vecA: int, vecB: int, ctas: int):
    totA, total = nm * vecA, nm * (vecA + vecB)
    stride = ctas * K_CHUNK
    done = [0] * nm
    last_chunk_end = {}  # (cta, job) -> end of the CTA's last chunk touching the job's A range
    flushes = []         # (cta, job, chunk index at flush)
    for b in range(ctas):
        pj, pc = -1, 0
        step = 0

        def flush():
            nonlocal pj, pc
            done[pj] += pc
            flushes.append((b, pj, step))
            pj, pc = -1, 0

        base = b * K_CHUNK
        while base < total:
            if base < totA:
                hi = min(base + K_CHUNK, totA)
                j0, j1 = base // vecA, (hi - 1) // vecA
                for j in range(j0, j1 + 1):
                    lo_j, hi_j = max(base, j * vecA), min(hi, (j + 1) * vecA)
                    last_chunk_end[(b, j)] = step
                    if pj != j:
                        if pj >= 0:
                            flush()
                        pj = j
                    pc += hi_j - lo_j
                    if j < j1:
                        flush()
                nxt = base + stride
                if pj >= 0 and (nxt >= totA or nxt >= (pj + 1) * vecA):
                    flush()
            base += stride
            step += 1
        if pj >= 0:
            flush()
    return done, last_chunk_end, flushes


@pytest.mark.parametrize("nm,vecA,vecB,ctas", [
    (1, 131104, 65552, 64),      # one miss, the decode shapes (W13+S13 / W2+S2 vectors)
    (3, 131104, 65552, 64),
    (8, 131104, 65552, 148),
    (64, 131104, 65552, 7),
    (5, 700, 300, 3),            # jobs smaller than a chunk: a chunk spans several jobs
    (9, 1024, 1024, 1),
    (2, 1, 1, 2),
])
def test_every_job_counted_exactly_once(nm, vecA, vecB, ctas):
    done, last, flushes = simulate(nm, vecA, vecB, ctas)
    assert done == [vecA] * nm
    # a CTA publishes a job once, at or after its last chunk of that job
    seen = set()
    for b, j, step in flushes:
        assert (b, j) not in seen
        seen.add((b, j))
        assert step >= last[(b, j)]
    assert seen == set(last)


def test_random_shapes():
    rng = random.Random(7)
    for _ in range(200):
        nm = rng.randint(1, 64)
        vecA = rng.randint(1, 5000)
        vecB = rng.randint(0, 3000)
        ctas = rng.randint(1, 300)
        done, _, _ = simulate(nm, vecA, vecB, ctas)
        assert done == [vecA] * nm, (nm, vecA, vecB, ctas)
