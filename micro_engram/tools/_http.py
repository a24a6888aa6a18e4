"""Minimal client of an OpenAI-compatible vLLM server (standard library only): the
completions endpoint with prompt log-probs, /tokenize and /v1/models."""
import json
import sys
import urllib.error
import urllib.request


class Server:
    def __init__(self, url, api_key=None, timeout=600.0):
        self.base = url.rstrip("/")
        self.headers = {"Content-Type": "application/json"}
        if api_key:
            self.headers["Authorization"] = f"Bearer {api_key}"
        self.timeout = timeout
        self._model = None

    def _open(self, req):
        try:
            return urllib.request.urlopen(req, timeout=self.timeout)
        except urllib.error.HTTPError as e:
            if e.code == 401:
                sys.exit("the server wants an API key: pass --api-key (or set VLLM_API_KEY)")
            raise
        except urllib.error.URLError as e:
            sys.exit(f"no server answered at {req.full_url} ({e.reason}): is vLLM up, on this host and port "
                     f"(--host 0.0.0.0 for another machine)?")

    def post(self, path, payload):
        req = urllib.request.Request(self.base + path, data=json.dumps(payload).encode(), headers=self.headers)
        with self._open(req) as r:
            return json.loads(r.read())

    def model(self, name=None):
        if name:
            self._model = name
        if self._model is None:
            req = urllib.request.Request(self.base + "/v1/models", headers=self.headers)
            with self._open(req) as r:
                self._model = json.loads(r.read())["data"][0]["id"]
        return self._model

    def tokenize(self, prompt=None, messages=None, add_special_tokens=None, add_generation_prompt=None):
        body = {"model": self.model()}
        if messages is not None:
            body["messages"] = messages
        else:
            body["prompt"] = prompt
        if add_special_tokens is not None:
            body["add_special_tokens"] = add_special_tokens
        if add_generation_prompt is not None:
            body["add_generation_prompt"] = add_generation_prompt
        return self.post("/tokenize", body)["tokens"]

    def prompt_logprobs(self, prompt, return_ids=False):
        """Per-position log-prob of the token that is actually there (no sampling)."""
        body = {"model": self.model(), "prompt": prompt, "max_tokens": 1, "temperature": 0, "prompt_logprobs": 0}
        if return_ids:
            body["return_token_ids"] = True
        return self.post("/v1/completions", body)["choices"][0]
