"""The decode attention under every kind of launch plan attn_prepare can choose: clusters of any size
up to 16 CTAs (the merge over a cluster's CTAs does not need a power of two), one or several clusters
per kv head (several merge through the scratch records), forced with YB_TUNE="acl=C,acs=S,acslots=N"
in a child process each (the tuning is read once per process; N, the slots per CTA of one cluster
before the kernel takes more clusters, set low so that the extra clusters are used).  Each child
checks yb_attention_dev against the CPU oracle of yalm's attention (src/infer.cpp:218-250) on a GQA
shape with a long cache and on two kv heads with a cache that several clusters share."""
import ctypes
import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SHAPES = [(32, 8, 128, 4096, 3232), (8, 2, 128, 8192, 6001), (8, 1, 64, 4096, 200)]


def _child(acl: int, acs: int, acslots: int) -> dict:
    import torch

    import oracle
    from yalm_b200 import _lib
    res = {}
    for nh, nkv, hd, msl, kv_len in SHAPES:
        rng = np.random.default_rng(kv_len + nh + acl + acslots)
        q = rng.standard_normal(nh * hd).astype(np.float32)
        k = rng.standard_normal((nkv, msl, hd), dtype=np.float32).astype(np.float16).view(np.uint16)
        v = rng.standard_normal((nkv, msl, hd), dtype=np.float32).astype(np.float16).view(np.uint16)
        scratch = torch.zeros(_lib.lib().yb_attention_scratch_bytes(nh, nkv, hd, msl), dtype=torch.uint8,
                              device="cuda")
        dq = torch.from_numpy(q).cuda()
        dk = torch.from_numpy(k).cuda()
        dv = torch.from_numpy(v).cuda()
        out = torch.zeros(nh * hd, dtype=torch.float32, device="cuda")
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        kb, vb = oracle.to_ref_kv_layout(k[:, :kv_len], v[:, :kv_len], msl)
        ref = oracle.mha(q, kb, vb, hd, kv_len, msl, nh, nkv)
        worst = 0.0
        for _ in range(2):  # the second call checks the merge counters were left at zero
            out.fill_(float("nan"))
            _lib.call("yb_attention_dev", p(out), p(dq), p(dk), p(dv), nh, nkv, hd, msl, kv_len, p(scratch), None)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            ok = bool(np.isfinite(got).all() and np.allclose(got, ref, rtol=1e-4, atol=2e-5))
            worst = max(worst, float(np.abs(got - ref).max()))
            if not ok:
                break
        info = (ctypes.c_int * 20)()
        _lib.call("yb_attention_plan_info", nh, nkv, hd, msl, info)
        res[f"{nh}/{nkv}/{hd}/{msl}/{kv_len}"] = {"ok": ok, "max_abs": worst, "cluster": info[0],
                                                   "clusters_per_kv_head": info[1]}
    return res


@pytest.mark.gpu
@pytest.mark.parametrize("acl,acs,acslots", [(16, 1, 1024), (12, 1, 1024), (10, 1, 1024), (7, 2, 256),
                                             (5, 3, 256), (3, 6, 1024), (1, 9, 128), (2, 32, 128)])
def test_attention_forced_plans_match_oracle(gpu, acl, acs, acslots):
    env = dict(os.environ, YB_TUNE=f"acl={acl},acs={acs},acslots={acslots}")
    r = subprocess.run([sys.executable, os.path.abspath(__file__), str(acl), str(acs), str(acslots)], cwd=ROOT,
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    for shape, d in res.items():
        assert d["cluster"] == acl, (shape, d)
        assert d["ok"], (shape, d)


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    print(json.dumps(_child(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]))))
