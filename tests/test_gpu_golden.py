"""The B200 engine against the reference's own outputs (tests/golden/*.npz):
same seeded checkpoint, prompt and fed tokens through ti_engine_prefill /
ti_engine_decode; logits within 2e-2 max-abs relative of the reference's."""
import glob
import json
import os
import sys

import numpy as np
import pytest

import oracle
import ti_b200 as ti

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
pytestmark = pytest.mark.gpu
FIXTURES = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))
TOL = 2e-2


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p)[:-4] for p in FIXTURES])
def test_engine_matches_reference_goldens(path):
    z = np.load(path)
    kw = json.loads(str(z["kw"]))
    lora = kw.pop("lora", None)
    eng = ti.Engine(ti.model_desc(**kw), max_batch=1, max_seq_len=64,
                    max_adapters=1 if lora else 0, max_lora_rank=lora["rank"] if lora else 0,
                    lora_proj_mask=lora["mask"] if lora else 0)
    eng.init_synthetic(int(z["seed"]), float(z["std"]))
    ad = -1
    if lora:
        ad = eng.adapter_create(lora["rank"], lora["alpha"], lora["mask"])
        eng.adapter_init_synthetic(ad, int(z["seed"]), lora["std_a"], lora["std_b"])
    sid = eng.seq_create()
    _, lb = eng.prefill(sid, z["prompt"], adapter=ad, logits=ti.LOGITS_BF16)
    rows = [oracle.bf16_to_f32(lb)]
    for t in z["feed"]:
        _, lb = eng.decode([sid], [int(t)], adapters=[ad] if lora else None, logits=ti.LOGITS_BF16)
        rows.append(oracle.bf16_to_f32(lb[0]))
    ref = z["ref_logits"]
    for i, g in enumerate(rows):
        err = np.abs(g - ref[i]).max() / np.abs(ref[i]).max()
        assert err <= TOL, (i, err)
    eng.check()
    eng.close()
