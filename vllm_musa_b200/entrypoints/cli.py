"""``b200-vllm`` command line: ``serve`` (OpenAI server), ``generate`` (one-shot offline run),
``collect-env`` (environment report), ``version``."""
from __future__ import annotations

import argparse
import json
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="b200-vllm")
    sub = ap.add_subparsers(dest="cmd", required=True)
    from .openai.api_server import make_arg_parser
    sp = sub.add_parser("serve", help="run the OpenAI-compatible server")
    sp.add_argument("model_tag", nargs="?", default=None)
    make_arg_parser(sp)
    gp = sub.add_parser("generate", help="generate from token ids / text")
    gp.add_argument("model")
    gp.add_argument("--prompt", default=None)
    gp.add_argument("--prompt-token-ids", default=None, help="comma-separated ids")
    gp.add_argument("--max-tokens", type=int, default=16)
    gp.add_argument("--temperature", type=float, default=0.0)
    gp.add_argument("--tensor-parallel-size", "-tp", type=int, default=1)
    gp.add_argument("--pipeline-parallel-size", "-pp", type=int, default=1)
    gp.add_argument("--device", default="cuda")
    sub.add_parser("collect-env", help="print the environment report")
    sub.add_parser("version")
    a = ap.parse_args(argv)
    if a.cmd == "serve":
        if a.model_tag:
            a.model = a.model_tag
        from .openai.api_server import run_server
        run_server(a)
    elif a.cmd == "generate":
        from .. import LLM, SamplingParams
        llm = LLM(a.model, tensor_parallel_size=a.tensor_parallel_size,
                  pipeline_parallel_size=a.pipeline_parallel_size, device=a.device)
        prompt = ([int(x) for x in a.prompt_token_ids.split(",")] if a.prompt_token_ids
                  else a.prompt)
        out = llm.generate([prompt], SamplingParams(temperature=a.temperature,
                                                    max_tokens=a.max_tokens))[0]
        print(json.dumps({"token_ids": out.outputs[0].token_ids, "text": out.outputs[0].text}))
        llm.shutdown()
    elif a.cmd == "collect-env":
        from ..collect_env import main as ce
        ce()
    else:
        from .. import __version__
        print(__version__)
    return 0


if __name__ == "__main__":
    sys.exit(main())
