"""Tensor-parallel decode on 2 GPUs (one process per GPU, the shape `bench.py --gpus 2` runs): each
rank holds half of the heads, FFN hidden units and vocabulary of the tiny checkpoint; the wo / w2
partial sums cross NVLink inside the matvec kernels.  Checked against yalm's CPU path: teacher-
forced logits at every step (max-abs <= 2e-2, cosine >= 0.9999), 64 free-running greedy ids equal to
the golden run, and bit-identical logits on every rank.  Skipped with fewer than 2 GPUs.

The ranks exchange only their IPC handles on the host (gloo); a rank that fails reports it through
its exit status and the parent bounds every wait."""
import os
import socket
import subprocess
import sys
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOGIT_MAX_ABS = 2e-2
LOGIT_COS = 0.9999


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank: int, world: int, port: int, path: str, out_dir: str) -> int:
    """One tensor-parallel rank: teacher-forced run over the golden stream, then a greedy run."""
    import datetime

    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from yalm_b200 import InferenceMode, InferenceState, Model, YALMData

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    g = dict(np.load(os.path.join(ROOT, "tests", "golden", "tiny_golden.npz")))
    m = Model(YALMData(path)).cuda(rank, rank, world)

    def all_gather(blob):
        out = [None] * world
        dist.all_gather_object(out, blob)
        return out

    m.tp_join(all_gather)
    s = InferenceState(m.config)
    seq = [int(t) for t in list(g["prompt"]) + list(g["greedy"])]
    forced = np.zeros((len(seq), m.config.vocab_size), np.float32)
    for pos, tok in enumerate(seq):
        m.forward(s, tok, pos, InferenceMode.OUTPUT_LOGITS)
        forced[pos] = s.logits()
    prompt = [int(t) for t in g["prompt"]]
    for pos, tok in enumerate(prompt):
        mode = InferenceMode.OUTPUT_LOGITS if pos + 1 == len(prompt) else InferenceMode.HYDRATE_KV_CACHE
        m.forward(s, tok, pos, mode)
    greedy = []
    for i in range(len(g["greedy"])):
        tok = int(np.argmax(s.logits()))
        greedy.append(tok)
        m.forward(s, tok, len(prompt) + i)
    status = m.status()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), forced=forced, greedy=np.array(greedy), status=status)
    dist.barrier()
    m.close()
    dist.destroy_process_group()
    return 0


@pytest.mark.gpu
def test_tp2_decode_matches_reference(gpu, tiny_yalm, golden):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import oracle
    world = 2
    port = _free_port()
    with tempfile.TemporaryDirectory() as out_dir:
        procs = [subprocess.Popen([sys.executable, os.path.abspath(__file__), str(r), str(world), str(port),
                                   tiny_yalm, out_dir], cwd=ROOT) for r in range(world)]
        rcs = []
        for p in procs:
            try:
                rcs.append(p.wait(timeout=600))
            except subprocess.TimeoutExpired:
                p.kill()
                rcs.append("timeout")
        assert rcs == [0] * world, rcs
        res = [dict(np.load(os.path.join(out_dir, f"rank{r}.npz"))) for r in range(world)]
    for r in range(world):
        assert int(res[r]["status"]) == 0
        assert np.array_equal(res[r]["forced"], res[0]["forced"]), f"rank {r} logits differ from rank 0"
        assert np.array_equal(res[r]["greedy"], res[0]["greedy"])
    ref = oracle.RefModel(tiny_yalm)
    seq = [int(t) for t in list(golden["prompt"]) + list(golden["greedy"])]
    worst = 0.0
    for pos, tok in enumerate(seq):
        exp = ref.forward(tok, pos, 1)
        got = res[0]["forced"][pos]
        d = float(np.abs(got - exp).max())
        worst = max(worst, d)
        cos = float(got @ exp / (np.linalg.norm(got) * np.linalg.norm(exp)))
        assert d <= LOGIT_MAX_ABS and cos >= LOGIT_COS, (pos, d, cos)
    assert [int(t) for t in res[0]["greedy"]] == [int(t) for t in golden["greedy"]]
    print("tp2 worst max-abs logit diff", worst)


if __name__ == "__main__":
    sys.exit(_rank_main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4], sys.argv[5]))
