"""A stand-in for vLLM's OpenAI server (the endpoints the runtime manager
uses): /health, /v1/models, /v1/load_lora_adapter, /v1/unload_lora_adapter.
Run as ``python fake_vllm_server.py HOST PORT``; loaded adapters are listed."""

import json
import sys
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

LORAS: dict[str, str] = {}


class H(BaseHTTPRequestHandler):
    def log_message(self, *a):  # quiet
        pass

    def _send(self, code, body):
        data = json.dumps(body).encode()
        self.send_response(code)
        self.send_header("content-type", "application/json")
        self.send_header("content-length", str(len(data)))
        self.end_headers()
        self.wfile.write(data)

    def do_GET(self):
        if self.path == "/health":
            return self._send(200, {})
        if self.path == "/v1/models":
            return self._send(200, {"data": [{"id": "base"}] + [{"id": k, "root": v} for k, v in LORAS.items()]})
        self._send(404, {})

    def do_POST(self):
        body = json.loads(self.rfile.read(int(self.headers.get("content-length", 0))) or b"{}")
        if self.path == "/v1/load_lora_adapter":
            if body["lora_name"] in LORAS:
                return self._send(400, {"error": "already loaded"})
            LORAS[body["lora_name"]] = body["lora_path"]
            return self._send(200, {})
        if self.path == "/v1/unload_lora_adapter":
            LORAS.pop(body["lora_name"], None)
            return self._send(200, {})
        self._send(404, {})


if __name__ == "__main__":
    ThreadingHTTPServer((sys.argv[1], int(sys.argv[2])), H).serve_forever()
