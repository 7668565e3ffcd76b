"""The drop-in, run inside yalm: yalm's own CLI (src/main.cpp) with yalm_b200/integration/yalm.patch
applied and yalm_b200/integration/b200.cpp added, linked to libyalm_b200.so (oracle/Makefile target
ref-b200, prebuilt into oracle/_ref/yalm_main_b200).  `-d b200` must print the same completion as
`-d cpu` — yalm's own tokenizer, prompt loop, greedy sampler and detokenizer around the engine —
and the same perplexity to float rounding."""
import os
import re
import subprocess

import pytest

import oracle
from yalm_b200 import synth

pytestmark = pytest.mark.gpu


def _run(args, timeout=600):
    env = dict(os.environ, OMP_NUM_THREADS=str(len(os.sched_getaffinity(0))))
    r = subprocess.run([oracle.YALM_MAIN_B200] + args, capture_output=True, text=True, timeout=timeout, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return r.stdout


def _completion(out: str) -> str:
    """The generated text: what run_completion prints between its encoding stats and its generation
    stats (src/main.cpp:178-190)."""
    m = re.search(r"Encoding stats:[^\n]*\n\n(.*?)\n\nGeneration stats:", out, re.S)
    assert m, out[-2000:]
    return m.group(1)


@pytest.fixture(scope="module")
def cli(gpu):
    if not os.path.exists(oracle.YALM_MAIN_B200):
        pytest.fail("oracle/_ref/yalm_main_b200 is not built (make -C oracle REF=<yalm checkout> ref-b200)")
    return oracle.YALM_MAIN_B200


@pytest.mark.parametrize("config,steps,context", [("tiny", 64, 0), ("tiny", 96, 64), ("mistral-7b", 32, 0)])
def test_cli_completion_b200_matches_cpu(cli, config, steps, context):
    """Greedy completion (-t 0) through yalm's CLI; context 64 runs the tiny model past its context
    (ring buffer and attention sinks)."""
    shape = synth.SHAPES[config]
    path = synth.write_yalm(os.path.join(synth.scratch_dir(synth.file_bytes(shape)), f"yalm_{config}_seed0.yalm"),
                            shape, seed=0)
    prompt = "~300~301~4000 hello ~777~1234"
    args = [path, "-t", "0", "-n", str(steps), "-i", prompt] + (["-T", str(context)] if context else [])
    cpu = _completion(_run(args + ["-d", "cpu"]))
    out = _run(args + ["-d", "b200"])
    assert "Using the yalm_b200 engine" in out
    b200 = _completion(out)
    assert b200 == cpu, f"cpu: {cpu!r}\nb200: {b200!r}"
    assert len(re.findall(r"~\d+", cpu)) >= min(steps, 16)


def test_cli_perplexity_b200_matches_cpu(cli):
    shape = synth.SHAPES["tiny"]
    path = synth.write_yalm(os.path.join(synth.scratch_dir(synth.file_bytes(shape)), "yalm_tiny_seed0.yalm"), shape,
                            seed=0)
    prompt = "".join(f"~{i}" for i in range(400, 600, 3))

    def ppl(dev):
        out = _run([path, "-m", "perplexity", "-i", prompt, "-d", dev])
        m = re.search(r"perplexity: ([0-9.eE+-]+)", out)
        assert m, out[-2000:]
        return float(m.group(1))

    a, b = ppl("cpu"), ppl("b200")
    assert abs(a - b) <= 1e-3 * a, (a, b)
