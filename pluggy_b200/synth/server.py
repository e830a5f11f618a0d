"""Local web front end: synthetic-corpus runs, training runs, model writing.

Parity: reference ``pluggy/synth/server.py:1-749`` (same pages, API paths and
request/response fields, so the reference's pages and scripts drive this server
too). Standard library only; it never imports torch on a page load.

    python -m pluggy_b200.synth.server [--host 127.0.0.1] [--port 8642]

Pages (a fixed allow-list, so no URL maps onto the file system):
``/`` corpus-config editor, ``/train`` training-run composer.

API (JSON unless noted)::

    GET  /api/meta                 styles, grounded modes, saved synth configs, uploads
    GET  /api/config/<name>        a saved config
    POST /api/config               {"name", "config"}: validate and save a synth config
    POST /api/upload?dataset=&filename=   raw body -> data/uploads/<dataset>/<stem>.jsonl
    POST /api/run | /api/stop      start / stop ``python -m pluggy_b200.synth.run``
    GET  /api/status               running, exit code, log tail, progress from the output dir
    GET  /api/train/meta           saved train configs, GPUs (nvidia-smi), registered models
    GET  /api/train/config/<name>  a saved train config
    POST /api/train/config         validate (against constructor signatures) and save
    POST /api/train/run            {"name", "steps": null|N}: torchrun over the local GPUs
    POST /api/train/stop           SIGTERM to the run's whole process group
    GET  /api/train/status         running, exit code, log tail, per-step metrics
    POST /api/model/write          {"name", "description", "kernels"}: model writer agent
    GET  /api/model/status         running, exit code, log tail, last phase, result

Each kind of run has its own slot (a :class:`Slot`): a subprocess with its log file.
Training runs start in their own session so that Stop reaches every rank; a run
outlives the server that started it.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import re
import signal
import socket
import subprocess
import sys
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from urllib.parse import parse_qs, urlparse

from pluggy_b200.synth.generate import STYLES
from pluggy_b200.synth.grounded import GROUNDED_MODES

STATIC = Path(__file__).parent / "static"
PKG_ROOT = Path(__file__).resolve().parents[1]
CONFIG_DIR = Path("configs")
UPLOAD_DIR = Path("data/uploads")
MAX_UPLOAD = 256 << 20
TAIL = 4000
MAX_POINTS = 400
SCAN_BYTES = 4 << 20

PAGES = {"/": "index.html", "/index.html": "index.html", "/train": "train.html",
         "/train.html": "train.html", "/theme.css": "theme.css", "/ui.js": "ui.js"}
MIME = {".html": "text/html; charset=utf-8", ".css": "text/css; charset=utf-8",
        ".js": "text/javascript; charset=utf-8"}

# the trainer's rank-0 line: step=N || loss=.. || gnorm=.. || lr=.. || tps=..
STEP_RE = re.compile(r"step=(\d+) \|\| loss=(\S+) \|\| gnorm=(\S+) \|\| lr=(\S+) \|\| tps=(\S+)")
RESULT_RE = re.compile(r"^RESULT (\{.*\})$", re.M)  # the model writer's last line
NAME_RE = re.compile(r"[A-Za-z0-9_\-]+")


class Slot:
    """One subprocess (a synth run, a training run or a model write) and its log."""

    def __init__(self):
        self.lock = threading.Lock()
        self.proc: subprocess.Popen | None = None
        self.log: Path | None = None
        self.meta: dict = {}

    def busy(self) -> bool:
        return self.proc is not None and self.proc.poll() is None

    def start(self, cmd: list[str], log: Path, header: str | None = None, session=False,
              **meta) -> None:
        with open(log, "w") as f:
            if header:
                f.write(header + "\n\n")
                f.flush()
            self.proc = subprocess.Popen(cmd, stdout=f, stderr=subprocess.STDOUT,
                                         env={**os.environ, "PYTHONUNBUFFERED": "1"},
                                         start_new_session=session)
        self.log, self.meta = log, meta

    def status(self) -> dict:
        st = {"running": False, "exit_code": None, "log_tail": ""}
        if self.proc is not None:
            code = self.proc.poll()
            st["running"], st["exit_code"] = code is None, code
        if self.log is not None and self.log.exists():
            st["log_tail"] = self.log.read_text(errors="replace")[-TAIL:]
        return st


SYNTH, TRAIN, WRITE = Slot(), Slot(), Slot()


# ---------------------------------------------------------------- helpers

def safe_name(name: str) -> str | None:
    name = name[:-5] if name.endswith(".json") else name
    return name if NAME_RE.fullmatch(name) else None


def _read_json(path: Path):
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, json.JSONDecodeError):
        return None


def is_synth_config(path: Path) -> bool:
    c = _read_json(path)
    return isinstance(c, dict) and ("seed_domains" in c or "grounding" in c)


def is_train_config(path: Path) -> bool:
    c = _read_json(path)
    return isinstance(c, dict) and "model" in c and "optimizer" in c


def saved(pred) -> list[str]:
    return sorted(p.stem for p in CONFIG_DIR.glob("*.json") if pred(p)) if CONFIG_DIR.exists() else []


def registered_models() -> list[str]:
    """Registry keys read from the builder's source (importing it would load torch)."""
    try:
        src = (PKG_ROOT / "models" / "builder.py").read_text()
    except OSError:
        return []
    m = re.search(r"MODEL_REGISTRY[^=]*=\s*\{(.*?)\n\}", src, re.S)
    keys = re.findall(r'"([^"]+)"\s*:', m.group(1)) if m else []
    gen = _read_json(PKG_ROOT / "models" / "generated" / "registry.json")
    return keys + sorted(gen) if isinstance(gen, dict) else keys


def gpus() -> list[str]:
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=10).stdout
    except (OSError, subprocess.SubprocessError):
        return []
    return [m.group(1) for m in re.finditer(r"GPU \d+: (.+?) \(UUID", out)]


def has_wandb() -> bool:
    return importlib.util.find_spec("wandb") is not None


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def normalize_upload(filename: str, body: bytes):
    """Document texts of an uploaded file, or an error string."""
    ext = Path(filename).suffix.lower()
    try:
        raw = body.decode("utf-8")
    except UnicodeDecodeError:
        return f"{filename}: not UTF-8 text (binary formats such as PDF are not supported)"

    def texts(rows):
        return [r if isinstance(r, str) else r["text"] for r in rows]

    try:
        if ext in (".txt", ".md"):
            docs = [raw]
        elif ext == ".jsonl":
            docs = texts(json.loads(x) for x in raw.splitlines() if x.strip())
        elif ext == ".json":
            rows = json.loads(raw)
            if not isinstance(rows, list):
                raise TypeError
            docs = texts(rows)
        else:
            return f"{filename}: unsupported extension {ext!r} (use .txt, .md, .jsonl or .json)"
    except (json.JSONDecodeError, KeyError, TypeError):
        return f"{filename}: rows must be strings or objects with a 'text' field"
    docs = [d.strip() for d in docs if isinstance(d, str) and d.strip()]
    return docs or f"{filename}: no non-empty documents"


def list_uploads() -> list[dict]:
    out = []
    if UPLOAD_DIR.exists():
        for ds in sorted(p for p in UPLOAD_DIR.iterdir() if p.is_dir()):
            docs = words = 0
            for fp in ds.glob("*.jsonl"):
                for line in fp.read_text(encoding="utf-8").splitlines():
                    if line.strip():
                        docs += 1
                        words += len(json.loads(line)["text"].split())
            out.append({"name": ds.name, "docs": docs, "words": words})
    return out


def validate_synth(cfg: dict) -> str | None:
    """First problem with a synth config (the checks ``run_pipeline`` would fail on)."""
    if cfg.get("provider") not in (None, "grok", "anthropic"):
        return "provider must be 'grok' or 'anthropic'"
    gen = cfg.get("generation", {})
    t = gen.get("temperature")
    if t is not None and (not isinstance(t, (int, float)) or not 0 <= t <= 2):
        return "generation.temperature must be a number in [0, 2]"
    dom, g = cfg.get("seed_domains"), cfg.get("grounding")
    if not dom and not g:
        return "set seed_domains (topic documents), grounding (uploaded text), or both"
    if dom is not None and not (isinstance(dom, list) and all(isinstance(d, str) and d.strip() for d in dom)):
        return "seed_domains must be a list of non-empty strings"
    if g is not None:
        if not isinstance(g.get("dir"), str):
            return "grounding.dir is required (e.g. data/uploads/<dataset>)"
        bad = [m for m in g.get("modes", []) if m not in GROUNDED_MODES]
        if bad:
            return f"unknown grounded modes: {bad}"
        if g.get("chunk_words", 600) < 50:
            return "grounding.chunk_words must be at least 50"
    if not isinstance(cfg.get("output", {}).get("dir"), str):
        return "output.dir is required"
    bad = [s for s in gen.get("styles", []) if s not in STYLES]
    if bad:
        return f"unknown styles: {bad}"
    q = cfg.get("quality", {})
    if q.get("enabled", True) and not 1 <= q.get("refine_min", 5) <= q.get("min_score", 7) <= 10:
        return "quality thresholds must satisfy 1 <= refine_min <= min_score <= 10"
    return None


def synth_progress(config_path: Path) -> dict:
    cfg = _read_json(config_path)
    try:
        out = Path(cfg["output"]["dir"])
    except (TypeError, KeyError):
        return {}
    prog = {"shards": len(list(out.glob("shard-*.jsonl")))}
    st = _read_json(out / "state.json")
    if isinstance(st, dict):
        prog["topics"] = len(st.get("topics") or [])
        prog["jobs_done"] = len(st.get("done", []))
    man = _read_json(out / "manifest.json")
    if man is not None:
        prog["manifest"] = man
    return prog


def validate_train(cfg: dict) -> str | None:
    """First problem with a train config: the trainer's own startup validation
    (structure, registries, constructor signatures as the schema), plus the checks
    that only matter for a launch from here. Imports torch lazily (on save/launch)."""
    if cfg.get("wandb", {}).get("enabled") and not has_wandb():
        return "wandb.enabled is set but wandb is not installed"
    from pluggy_b200.train.validate import ConfigError, validate_config

    try:
        validate_config(cfg)
    except ConfigError as e:
        return str(e)
    return None


def train_metrics(log: Path) -> list[dict]:
    try:
        text = log.read_text(errors="replace")[-SCAN_BYTES:]
    except OSError:
        return []
    pts = [{"step": int(m[1]), "loss": float(m[2]), "gnorm": float(m[3]), "lr": float(m[4]),
            "tps": float(m[5])} for m in STEP_RE.finditer(text)]
    if len(pts) <= MAX_POINTS:
        return pts
    stride = len(pts) // MAX_POINTS + 1
    return pts[::stride] + [pts[-1]]  # the last point feeds the status line


# ---------------------------------------------------------------- handlers

class Handler(BaseHTTPRequestHandler):
    def log_message(self, fmt, *args):  # the terminal belongs to the runs
        pass

    def send(self, code: int, body: bytes, ctype: str) -> None:
        self.send_response(code)
        self.send_header("Content-Type", ctype)
        self.send_header("Content-Length", str(len(body)))
        self.end_headers()
        self.wfile.write(body)

    def ok(self, obj, code: int = 200) -> None:
        self.send(code, json.dumps(obj).encode(), "application/json")

    def err(self, msg: str, code: int = 400) -> None:
        self.ok({"error": msg}, code)

    # GET -------------------------------------------------------------------
    def do_GET(self):
        path = urlparse(self.path).path
        if path in PAGES:
            name = PAGES[path]
            return self.send(200, (STATIC / name).read_bytes(), MIME[Path(name).suffix])
        route = {"/api/meta": self.get_meta, "/api/status": self.get_status,
                 "/api/train/meta": self.get_train_meta, "/api/train/status": self.get_train_status,
                 "/api/model/status": self.get_model_status}.get(path)
        if route is not None:
            return route()
        for prefix in ("/api/config/", "/api/train/config/"):
            if path.startswith(prefix):
                name = safe_name(path[len(prefix):])
                cfg = _read_json(CONFIG_DIR / f"{name}.json") if name else None
                return self.ok(cfg) if cfg is not None else self.err("config not found", 404)
        self.err("not found", 404)

    def get_meta(self):
        self.ok({"styles": STYLES, "grounded_modes": GROUNDED_MODES,
                 "configs": saved(is_synth_config), "uploads": list_uploads()})

    def get_status(self):
        with SYNTH.lock:
            st = SYNTH.status()
            cfg = SYNTH.meta.get("config")
        st["config"] = str(cfg) if cfg else None
        st["progress"] = synth_progress(cfg) if cfg else {}
        self.ok(st)

    def get_train_meta(self):
        g = gpus()
        self.ok({"configs": saved(is_train_config), "gpus": g, "gpu_count": len(g),
                 "models": registered_models(), "wandb": has_wandb()})

    def get_train_status(self):
        with TRAIN.lock:
            st = TRAIN.status()
            cfg, steps = TRAIN.meta.get("config"), TRAIN.meta.get("steps")
        st.update(config=str(cfg) if cfg else None, steps=steps, total_steps=None, metrics=[])
        c = _read_json(cfg) if cfg else None
        if c is not None:
            try:
                st["total_steps"] = steps or c["optimizer"]["scheduler"]["total_steps"]
            except (KeyError, TypeError):
                pass
        if TRAIN.log is not None:
            st["metrics"] = train_metrics(TRAIN.log)
        self.ok(st)

    def get_model_status(self):
        with WRITE.lock:
            st = WRITE.status()
            st["name"] = WRITE.meta.get("name")
        st["result"] = None
        if WRITE.log is not None and WRITE.log.exists():
            text = WRITE.log.read_text(errors="replace")
            lines = [x for x in text.splitlines() if x.strip()]
            st["phase"] = lines[-1][:200] if lines else ""
            m = RESULT_RE.search(text)
            if m:
                try:
                    st["result"] = json.loads(m.group(1))
                except json.JSONDecodeError:
                    pass
        self.ok(st)

    # POST ------------------------------------------------------------------
    def do_POST(self):
        path = urlparse(self.path).path
        if path == "/api/upload":
            return self.upload()
        try:
            n = int(self.headers.get("Content-Length", 0))
            body = json.loads(self.rfile.read(n) or b"{}")
        except (ValueError, json.JSONDecodeError):
            return self.err("invalid JSON body")
        if not isinstance(body, dict):
            return self.err("the body must be a JSON object")
        route = {"/api/config": lambda b: self.save(b, validate_synth),
                 "/api/train/config": lambda b: self.save(b, validate_train),
                 "/api/run": self.synth_run, "/api/stop": self.synth_stop,
                 "/api/train/run": self.train_run, "/api/train/stop": self.train_stop,
                 "/api/model/write": self.model_write}.get(path)
        if route is None:
            return self.err("not found", 404)
        route(body)

    def save(self, body, validate):
        name = safe_name(str(body.get("name", "")))
        if name is None:
            return self.err("name must match [A-Za-z0-9_-]+")
        cfg = body.get("config")
        problem = validate(cfg) if isinstance(cfg, dict) else "config must be an object"
        if problem:
            return self.err(problem)
        CONFIG_DIR.mkdir(exist_ok=True)
        path = CONFIG_DIR / f"{name}.json"
        with open(path, "w") as f:
            json.dump(cfg, f, indent=2)
        self.ok({"saved": str(path)})

    def _config_path(self, body) -> Path | None:
        name = safe_name(str(body.get("name", "")))
        path = CONFIG_DIR / f"{name}.json" if name else None
        return path if path is not None and path.exists() else None

    def synth_run(self, body):
        path = self._config_path(body)
        if path is None:
            return self.err("config not found; save it first", 404)
        with SYNTH.lock:
            if SYNTH.busy():
                return self.err("a run is already in progress", 409)
            log = Path(f"synth_run_{path.stem}.log")
            SYNTH.start([sys.executable, "-m", "pluggy_b200.synth.run", "--config", str(path)], log,
                        config=path)
        self.ok({"started": str(path), "log": str(log)})

    def synth_stop(self, body):
        with SYNTH.lock:
            if not SYNTH.busy():
                return self.err("no run in progress", 409)
            SYNTH.proc.terminate()
        self.ok({"stopped": True})

    def train_run(self, body):
        path = self._config_path(body)
        if path is None:
            return self.err("config not found; save it first", 404)
        cfg = _read_json(path)
        problem = validate_train(cfg) if isinstance(cfg, dict) else "config is not a JSON object"
        if problem:
            return self.err(problem)
        steps = body.get("steps")
        if steps is not None and (not isinstance(steps, int) or isinstance(steps, bool) or steps < 1):
            return self.err("steps must be a positive integer or null")
        nproc = 1
        for v in cfg["mesh"].values():
            nproc *= v
        g = gpus()
        if not g:
            return self.err("no CUDA GPUs visible to the server (nvidia-smi lists none)", 409)
        if nproc > len(g):
            return self.err(f"the mesh needs {nproc} ranks but this machine has {len(g)} GPU(s)", 409)
        with TRAIN.lock:
            if TRAIN.busy():
                return self.err("a training run is already in progress", 409)
            log = Path(f"train_run_{path.stem}.log")
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                   f"--nproc_per_node={nproc}", "--master_addr=127.0.0.1",
                   f"--master_port={free_port()}", "-m", "pluggy_b200.train.train",
                   "--config", str(path)]
            if steps is not None:
                cmd += ["--steps", str(steps)]
            TRAIN.start(cmd, log, header=" ".join(cmd), session=True, config=path, steps=steps)
        self.ok({"started": str(path), "log": str(log), "nproc": nproc, "steps": steps,
                 "cmd": " ".join(cmd)})

    def train_stop(self, body):
        with TRAIN.lock:
            if not TRAIN.busy():
                return self.err("no training run in progress", 409)
            # the run has its own session: signal the launcher and every rank
            os.killpg(os.getpgid(TRAIN.proc.pid), signal.SIGTERM)
        self.ok({"stopped": True})

    def model_write(self, body):
        name = str(body.get("name", ""))
        if not re.fullmatch(r"[A-Za-z0-9_]+", name):
            return self.err("name must match [A-Za-z0-9_]+ (it becomes a module name)")
        desc = str(body.get("description") or "").strip()
        if len(desc) < 20:
            return self.err("describe the architecture in a sentence or two: layers, widths, "
                            "attention layout, anything unusual")
        if "XAI_API_KEY" not in os.environ and not body.get("provider") == "anthropic":
            return self.err("XAI_API_KEY is not set in the server's environment", 409)
        target = PKG_ROOT / "models" / "generated" / f"{name}.py"
        if target.exists() and not body.get("overwrite"):
            return self.err(f"{target} already exists; pick another name", 409)
        with WRITE.lock:
            if WRITE.busy():
                return self.err("already writing a model", 409)
            log = Path(f"write_model_{name}.log")
            cmd = [sys.executable, "-m", "pluggy_b200.synth.write_model", "--name", name,
                   "--description", desc]
            if not body.get("kernels", True):
                cmd.append("--no-kernels")
            if body.get("overwrite"):
                cmd.append("--overwrite")
            WRITE.start(cmd, log, name=name)
        self.ok({"started": name, "log": str(log)})

    def upload(self):
        q = parse_qs(urlparse(self.path).query)
        ds = safe_name(q.get("dataset", [""])[0])
        if ds is None:
            return self.err("dataset must match [A-Za-z0-9_-]+")
        fname = Path(q.get("filename", [""])[0]).name
        if not fname:
            return self.err("the filename query parameter is required")
        n = int(self.headers.get("Content-Length", 0))
        if n <= 0:
            return self.err("empty upload")
        if n > MAX_UPLOAD:
            return self.err(f"uploads are limited to {MAX_UPLOAD >> 20} MiB", 413)
        docs = normalize_upload(fname, self.rfile.read(n))
        if isinstance(docs, str):
            return self.err(docs)
        out = UPLOAD_DIR / ds
        out.mkdir(parents=True, exist_ok=True)
        stem = re.sub(r"[^A-Za-z0-9_\-]", "_", Path(fname).stem) or "upload"
        path = out / f"{stem}.jsonl"
        with open(path, "w", encoding="utf-8") as f:
            f.writelines(json.dumps({"text": d}, ensure_ascii=False) + "\n" for d in docs)
        self.ok({"saved": str(path), "docs": len(docs), "words": sum(len(d.split()) for d in docs),
                 "grounding_dir": str(out)})


def make_server(host: str = "127.0.0.1", port: int = 8642) -> ThreadingHTTPServer:
    return ThreadingHTTPServer((host, port), Handler)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="local front end for corpus and training runs")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8642)
    a = p.parse_args(argv)
    srv = make_server(a.host, a.port)
    print(f"front end: http://{a.host}:{a.port}")
    try:
        srv.serve_forever()
    except KeyboardInterrupt:
        srv.shutdown()


if __name__ == "__main__":
    main()
