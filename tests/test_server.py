"""Front-end server: pages, config CRUD and validation, uploads, run slots, metrics."""

import json
import threading
import urllib.error
import urllib.request

import pytest

from pluggy_b200.synth import server as srv


@pytest.fixture()
def base(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    s = srv.make_server("127.0.0.1", 0)
    t = threading.Thread(target=s.serve_forever, daemon=True)
    t.start()
    yield f"http://127.0.0.1:{s.server_address[1]}"
    s.shutdown()


def call(url, body=None, raw=None):
    data = raw if raw is not None else (json.dumps(body).encode() if body is not None else None)
    req = urllib.request.Request(url, data=data, method="POST" if data is not None else "GET")
    try:
        with urllib.request.urlopen(req, timeout=30) as r:
            return r.status, r.read()
    except urllib.error.HTTPError as e:
        return e.code, e.read()


def js(url, body=None, raw=None):
    code, b = call(url, body, raw)
    return code, json.loads(b)


SYNTH = {"seed_domains": ["physics"], "output": {"dir": "data/out"},
         "generation": {"styles": ["textbook"]}}

TRAIN = {"run_name": "t", "mesh": {"dp": 1}, "parallelism": "ddp",
         "model": {"name": "qwen3_dense", "config": {"num_layers": 2, "num_heads": 4, "num_kv_heads": 2,
                                                     "emb_dim": 64, "head_dim": 16, "vocab_size": 128,
                                                     "ffn_dim": 128}},
         "optimizer": {"name": "adamw", "config": {"lr": 1e-3},
                       "scheduler": {"type": "cosine", "total_steps": 10, "warmup_ratio": 0.1}},
         "objective": {"name": "AR", "config": {}},
         "data": {"synthetic": {"s": 1.1}, "seq_len": 64, "global_batch_size": 4, "micro_batch_size": 2}}


def test_pages_allowlist(base):
    for p in ("/", "/train", "/theme.css", "/ui.js"):
        code, body = call(base + p)
        assert code == 200 and len(body) > 100
    assert call(base + "/../server.py")[0] == 404
    assert call(base + "/static/ui.js")[0] == 404


def test_synth_config_crud(base):
    code, meta = js(base + "/api/meta")
    assert code == 200 and "textbook" in meta["styles"] and "qa" in meta["grounded_modes"]
    assert js(base + "/api/config", {"name": "bad/name", "config": SYNTH})[0] == 400
    code, r = js(base + "/api/config", {"name": "s1", "config": {**SYNTH, "provider": "x"}})
    assert code == 400 and "provider" in r["error"]
    code, r = js(base + "/api/config", {"name": "s1", "config": {
        **SYNTH, "quality": {"min_score": 4, "refine_min": 6}}})
    assert code == 400 and "refine_min" in r["error"]
    assert js(base + "/api/config", {"name": "s1", "config": SYNTH})[0] == 200
    code, cfg = js(base + "/api/config/s1")
    assert code == 200 and cfg == SYNTH
    assert js(base + "/api/meta")[1]["configs"] == ["s1"]
    assert js(base + "/api/config/nope")[0] == 404
    assert js(base + "/api/stop", {})[0] == 409  # nothing running
    st = js(base + "/api/status")[1]
    assert st["running"] is False and st["exit_code"] is None


def test_upload_normalisation(base):
    u = base + "/api/upload?dataset=docs&filename="
    code, r = js(u + "a.md", raw="# Title\n\nBody text here.".encode())
    assert code == 200 and r["docs"] == 1 and r["grounding_dir"].endswith("docs")
    code, r = js(u + "b.jsonl", raw=b'{"text": "one two"}\n"three"\n\n')
    assert code == 200 and r["docs"] == 2 and r["words"] == 3
    assert js(u + "c.json", raw=b'{"text": "x"}')[0] == 400  # not a list
    assert js(u + "d.pdf", raw=b"%PDF")[0] == 400
    assert js(u + "e.txt", raw=b"\xff\xfe")[0] == 400
    assert js(base + "/api/upload?dataset=../x&filename=a.txt", raw=b"hi")[0] == 400
    meta = js(base + "/api/meta")[1]
    assert meta["uploads"] == [{"name": "docs", "docs": 3, "words": 8}]
    rows = [json.loads(x) for x in open("data/uploads/docs/b.jsonl")]
    assert rows == [{"text": "one two"}, {"text": "three"}]


def test_train_config_validation(base):
    ok = js(base + "/api/train/config", {"name": "t1", "config": TRAIN})
    assert ok[0] == 200, ok
    bad_key = json.loads(json.dumps(TRAIN))
    bad_key["model"]["config"]["hidden"] = 3
    code, r = js(base + "/api/train/config", {"name": "t2", "config": bad_key})
    assert code == 400 and "unknown argument" in r["error"] and "hidden" in r["error"]
    missing = json.loads(json.dumps(TRAIN))
    del missing["model"]["config"]["vocab_size"]
    code, r = js(base + "/api/train/config", {"name": "t2", "config": missing})
    assert code == 400 and "missing required argument" in r["error"]
    div = json.loads(json.dumps(TRAIN))
    div["data"]["global_batch_size"] = 3
    assert "divisible" in js(base + "/api/train/config", {"name": "t2", "config": div})[1]["error"]
    nosched = json.loads(json.dumps(TRAIN))
    nosched["optimizer"]["scheduler"]["type"] = "linear"
    assert "scheduler" in js(base + "/api/train/config", {"name": "t2", "config": nosched})[1]["error"]
    meta = js(base + "/api/train/meta")[1]
    assert meta["configs"] == ["t1"] and "qwen3_dense" in meta["models"]
    assert js(base + "/api/train/run", {"name": "t1", "steps": 0})[0] == 400
    assert js(base + "/api/train/stop", {})[0] == 409


def test_train_metrics_parsing(tmp_path):
    log = tmp_path / "l.log"
    log.write_text("\n".join(f"step={i} || loss={10 - i * 0.01:.4f} || gnorm=1.000 || lr=3.00e-04 "
                             f"|| tps={1000 + i}" for i in range(1000)))
    pts = srv.train_metrics(log)
    assert len(pts) <= srv.MAX_POINTS + 1 and pts[-1]["step"] == 999 and pts[0]["step"] == 0


def test_model_write_checks(base, monkeypatch):
    monkeypatch.delenv("XAI_API_KEY", raising=False)
    assert js(base + "/api/model/write", {"name": "a-b", "description": "x" * 40})[0] == 400
    assert js(base + "/api/model/write", {"name": "ab", "description": "short"})[0] == 400
    assert js(base + "/api/model/write", {"name": "ab", "description": "x" * 40})[0] == 409
    st = js(base + "/api/model/status")[1]
    assert st["running"] is False and st["result"] is None
