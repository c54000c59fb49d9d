"""Loopback completion server over this framework's block-diffusion decoder (the engine the
weight-space bench talks to; the reference runs llama.cpp's llama-server in this role).

    python -m dllm_qwen38_b200.weight_space.server --model HF_DIR|PRESET [--tokenizer HF_DIR|bytes]
           [--port 17977] [--block 32] [--threshold 0.9] [--sub-block 0] [--n-ctx 8192]

Endpoints (JSON):
  GET  /health      {"status": "ok"} once the model is loaded
  GET  /props       {"model_path", "default_generation_settings": {"n_ctx"}, "decoder": {...},
                     "engine": "dllm_qwen38_b200"}
  POST /completion  {"prompt": str, "n_predict": int, "temperature": 0.0, ...} ->
                    {"content", "tokens_predicted", "stop_type": "eos" | "limit", "stopped_limit",
                     "stopped_eos", "timings": {"predicted_ms", "forwards"}}
Decoding is greedy (temperature 0) confidence-threshold block diffusion through the cached block
decoder (`infer/cached.py`); any other temperature is refused. The server binds 127.0.0.1 only
and serves one request at a time. `--tokenizer bytes` is a byte-level tokenizer (ids 3..258, EOS
2) for presets without a vocabulary file.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import torch

MAX_BODY = 1 << 20


class ByteTokenizer:
    """UTF-8 bytes as ids 3..258; 2 is EOS."""

    eos_token_id = 2

    def encode(self, text: str) -> list:
        return [b + 3 for b in text.encode("utf-8")]

    def decode(self, ids) -> str:
        return bytes(i - 3 for i in ids if 3 <= i < 259).decode("utf-8", errors="replace")


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path)
        self.eos_token_id = self.tok.eos_token_id

    def encode(self, text: str) -> list:
        return list(self.tok(text, add_special_tokens=False)["input_ids"])

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)


class Engine:
    def __init__(self, model_spec: str, tokenizer: str, block: int, threshold: float, sub_block: int, n_ctx: int,
                 ckpt: str | None = None):
        from ..native_tools import api

        self.model = api.load(model_spec)
        if ckpt:
            from safetensors.torch import load_file

            from ..io import ckpt as ck

            ck.restore_into(self.model, load_file(ckpt), ctx=ckpt)
        self.tok = ByteTokenizer() if tokenizer == "bytes" else HFTokenizer(tokenizer)
        self.block, self.threshold, self.sub_block, self.n_ctx = block, threshold, sub_block or None, n_ctx
        self.model_path = str(pathlib.Path(model_spec).resolve()) if os.path.exists(model_spec) else model_spec
        self.lock = threading.Lock()

    def props(self) -> dict:
        return {"model_path": self.model_path, "engine": "dllm_qwen38_b200",
                "default_generation_settings": {"n_ctx": self.n_ctx},
                "decoder": {"kind": "block-diffusion", "block": self.block, "threshold": self.threshold,
                            "sub_block": self.sub_block or 0}}

    @torch.no_grad()
    def complete(self, req: dict) -> dict:
        from ..infer.cached import generate

        prompt = req.get("prompt")
        n_predict = req.get("n_predict", 128)
        if not isinstance(prompt, str) or not prompt:
            raise ValueError("prompt must be a non-empty string")
        if type(n_predict) is not int or n_predict < 1:
            raise ValueError("n_predict must be a positive integer")
        if float(req.get("temperature", 0.0)) != 0.0:
            raise ValueError("only greedy decoding (temperature 0) is served")
        ids = self.tok.encode(prompt)
        if len(ids) + n_predict + self.block > self.n_ctx:
            raise ValueError("prompt + n_predict exceeds n_ctx")
        cfg = self.model.config
        eos = self.tok.eos_token_id
        n_blocks = -(-(len(ids) % self.block + n_predict) // self.block)
        t0 = time.perf_counter()
        with self.lock:
            tr = generate(self.model, ids, n_blocks=n_blocks, block=self.block, mask_id=cfg.mask_id,
                          threshold=self.threshold, sub_block=self.sub_block, eos_id=eos, temperature=0.0)
            if torch.cuda.is_available():
                torch.cuda.synchronize()
        ms = (time.perf_counter() - t0) * 1e3
        gen = tr.tokens[len(ids):]
        stopped_eos = eos is not None and eos in gen
        if stopped_eos:
            gen = gen[:gen.index(eos)]
        gen = gen[:n_predict]
        return {"content": self.tok.decode(gen), "tokens_predicted": len(gen),
                "stop_type": "eos" if stopped_eos else "limit", "stopped_eos": stopped_eos,
                "stopped_limit": not stopped_eos, "timings": {"predicted_ms": ms, "forwards": tr.forwards}}


def make_handler(engine: Engine):
    class Handler(BaseHTTPRequestHandler):
        def log_message(self, *args):  # quiet
            pass

        def _send(self, code: int, body: dict):
            data = json.dumps(body).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            if self.path == "/health":
                self._send(200, {"status": "ok"})
            elif self.path == "/props":
                self._send(200, engine.props())
            else:
                self._send(404, {"error": "not found"})

        def do_POST(self):
            if self.path != "/completion":
                self._send(404, {"error": "not found"})
                return
            n = int(self.headers.get("Content-Length", "0"))
            if n <= 0 or n > MAX_BODY:
                self._send(413, {"error": "body size"})
                return
            try:
                req = json.loads(self.rfile.read(n))
                self._send(200, engine.complete(req))
            except ValueError as e:
                self._send(400, {"error": str(e)})

    return Handler


def serve(engine: Engine, port: int) -> ThreadingHTTPServer:
    return ThreadingHTTPServer(("127.0.0.1", port), make_handler(engine))


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", required=True)
    p.add_argument("--ckpt", default=None, help="safetensors weights to load over the model")
    p.add_argument("--tokenizer", default=None, help="HF tokenizer dir, or 'bytes' (default: the model dir)")
    p.add_argument("--port", type=int, default=17977)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--threshold", type=float, default=0.9)
    p.add_argument("--sub-block", type=int, default=0)
    p.add_argument("--n-ctx", type=int, default=8192)
    a = p.parse_args(argv)
    tok = a.tokenizer or (a.model if os.path.isdir(a.model) else "bytes")
    eng = Engine(a.model, tok, a.block, a.threshold, a.sub_block, a.n_ctx, a.ckpt)
    srv = serve(eng, a.port)
    print(json.dumps({"listening": f"http://127.0.0.1:{a.port}", **eng.props()}), flush=True)
    try:
        srv.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        srv.server_close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
