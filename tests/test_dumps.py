"""CPU: logit-dump and token-id files in the reference's -DDUMP_LOGITS formats
(raw fp32 rows appended per step; a JSON id list), read back the way the
reference's analysis script reads them (raw float32 reshaped to (steps,
vocab), .npy as stored, json.load for ids)."""
import json

import numpy as np


def test_raw_dump_round_trip(pkg, tmp_path):
    d = pkg.dumps
    rng = np.random.default_rng(3)
    steps = [rng.normal(0, 2, 32000).astype(np.float32) for _ in range(5)]
    path = tmp_path / "ours.bin"
    d.append_logits(path, steps[0], first=True)
    for s in steps[1:3]:
        d.append_logits(path, s)
    d.append_logits(path, np.stack(steps[3:]))
    raw = np.frombuffer(path.read_bytes(), dtype=np.float32)  # the analysis script's read
    assert raw.size == 5 * 32000
    assert np.array_equal(raw.reshape(5, 32000), np.stack(steps))
    assert np.array_equal(d.load_logits(path, 32000), np.stack(steps))
    d.append_logits(path, steps[0], first=True)  # step 0 truncates, as "wb" does
    assert d.load_logits(path, 32000).shape == (1, 32000)


def test_npy_dump(pkg, tmp_path):
    x = np.random.default_rng(4).normal(0, 1, (3, 100)).astype(np.float32)
    pkg.dumps.save_logits_npy(tmp_path / "ours.npy", x)
    assert np.array_equal(np.load(tmp_path / "ours.npy"), x)
    assert np.array_equal(pkg.dumps.load_logits(str(tmp_path / "ours.npy"), 100), x)


def test_token_ids_json(pkg, tmp_path):
    d = pkg.dumps
    p = tmp_path / "ids.json"
    d.append_token_ids(p, [29892, 727], first=True)
    d.append_token_ids(p, np.array([471, 263], np.int32))
    assert json.loads(p.read_text()) == [29892, 727, 471, 263]
    p.write_text("[1,2,3")  # the reference's writer leaves the list open
    assert d.load_token_ids(p) == [1, 2, 3]
