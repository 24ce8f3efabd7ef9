"""The continuous-batching scheduler of the driver's "batch" verb
(llm-inference-diy_b200/csrc/batch_sched.h) on the CPU, against a fake model (tests/native/
sched_harness.cpp): every request must get exactly what a turn of its own would produce
(QwenEngine turn loop, framework_src/qwen_infer.cu:786-818: prefill prompt[:-1], steps from
prompt[-1] at position n-1, stop ids not printed, a token limit), with at most `slots` requests
in flight, FIFO admission into the lowest free slot, and rejected prompts reported."""
import os
import random
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "llm-inference-diy_b200", "csrc")
STOP = (151645, 151643)


def fake_next(t, p):
    if (t + 3 * p) % 23 == 0:
        return 151645
    return (t * 31 + p * 7 + 3) % 997


@pytest.fixture(scope="module")
def harness():
    d = tempfile.mkdtemp()
    exe = os.path.join(d, "sched_harness")
    subprocess.run(["g++", "-O1", "-std=c++17", "-I", CSRC, "-o", exe, os.path.join(HERE, "native", "sched_harness.cpp")],
                   check=True)
    yield exe
    os.remove(exe)


def run(exe, slots, max_len, max_new, stop, vocab, reqs, env=None):
    text = f"{slots} {max_len} {max_new} {int(stop)} {vocab}\n" + "".join(" ".join(map(str, r)) + "\n" for r in reqs)
    text += "end\n"
    p = subprocess.run([exe], input=text, capture_output=True, text=True, check=True, env=env)
    return [l.split() for l in p.stdout.splitlines()]


def single_turn(prompt, max_len, max_new, stop, vocab):
    """What one turn of its own produces for a prompt (None = rejected)."""
    n = len(prompt)
    if n < 1 or n > max_len or any(not 0 <= t < vocab for t in prompt):
        return None
    limit = min(max_new, max_len - n + 1)
    out, tok, pos = [], prompt[-1], n - 1
    for _ in range(limit):
        t = fake_next(tok, pos)
        if stop and t in STOP:
            break
        out.append(t)
        tok, pos = t, pos + 1
    return out


@pytest.mark.parametrize("slots,max_new,stop", [(1, 20, True), (3, 20, True), (4, 60, False), (16, 40, True)])
def test_streams_match_single_turns(harness, slots, max_new, stop):
    rng = random.Random(slots * 100 + max_new)
    vocab, max_len = 151936, 64  # the stop ids are ordinary tokens when stop is off
    reqs = [[rng.randrange(1000) for _ in range(rng.randint(1, 30))] for _ in range(11)]
    reqs[3] = []                    # empty: rejected
    reqs[5] = [5, vocab + 2, 7]     # id out of range: rejected
    reqs[7] = list(range(max_len))  # exactly max_len: one step at position max_len-1
    reqs[8] = list(range(max_len + 1))  # too long: rejected
    ev = run(harness, slots, max_len, max_new, stop, vocab, reqs)
    assert ev[-1] == ["RC", "0"]
    got = {r: [] for r in range(len(reqs))}
    done, active, peak, order = {}, set(), 0, []
    slot_of = {}
    for e in ev[:-1]:
        if e[0] == "P":
            continue
        if e[0] == "S":
            B = int(e[1])
            assert 1 <= B <= slots
            for i, tp in enumerate(e[2:]):
                t, p = map(int, tp.split(":"))
                assert 0 <= p < max_len and 0 <= t < vocab
        elif e[0] == "E":
            r = int(e[1])
            assert r not in done
            if r not in active:
                active.add(r)
                order.append(r)
            peak = max(peak, len(active))
            got[r].append(int(e[2]))
        elif e[0] == "D":
            r = int(e[1])
            assert r not in done
            done[r] = int(e[2])
            active.discard(r)
    assert sorted(done) == list(range(len(reqs)))
    assert peak <= slots
    for r, p in enumerate(reqs):
        want = single_turn(p, max_len, max_new, stop, vocab)
        if want is None:
            assert done[r] == 2 and got[r] == [], r
        else:
            assert got[r] == want, (r, got[r], want)
            assert done[r] in (0, 1)
    # admission is first come, first served
    assert order == sorted(order)


def test_prefill_and_positions(harness):
    """Prompt rows 0..n-2 are prefilled into the request's slot; its first step is at position n-1."""
    ev = run(harness, 2, 32, 3, False, 1000, [[1, 2, 3, 4], [9], [7, 8]])
    pre = [(int(e[1]), int(e[2])) for e in ev if e[0] == "P"]
    assert pre[0] == (0, 3)  # request 0 in slot 0, three prompt rows
    assert (0, 1) in pre     # request 2 later takes a free slot (request 1 had a one-token prompt: no prefill)
    first = next(e for e in ev if e[0] == "S")
    assert first[1] == "2" and first[2] == "4:3" and first[3] == "9:0"


def test_callback_failure_stops_the_run(harness):
    ev = run(harness, 2, 32, 10, False, 1000, [[1, 2], [3]], env=dict(os.environ, FAIL_AFTER="2"))
    assert ev[-1] == ["RC", "7"]
    assert not any(e[0] == "D" for e in ev)  # unfinished requests get no done()
