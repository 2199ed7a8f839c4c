"""Command line of the runtime.

    python -m vllm_sm70_b200 serve --model CKPT [--port 8000 ...]    # OpenAI server
    python -m vllm_sm70_b200 convert-gguf model.gguf OUT [...]        # GGUF -> HF safetensors
    python -m vllm_sm70_b200 eval-envelope --model CKPT [...]         # teacher-forced noise floor

Each subcommand forwards its remaining arguments to the module that owns it
(``entrypoints.openai_server``, ``models.convert_gguf``,
``eval.teacher_forced``); ``<subcommand> --help`` lists them.
"""
from __future__ import annotations

import sys

COMMANDS = {
    "serve": ("vllm_sm70_b200.entrypoints.openai_server", "OpenAI-compatible HTTP server"),
    "convert-gguf": ("vllm_sm70_b200.models.convert_gguf", "GGUF -> HF safetensors"),
    "eval-envelope": ("vllm_sm70_b200.eval.teacher_forced",
                      "teacher-forced log-prob envelope between two chunkings"),
}


def main(argv=None) -> int:
    import importlib

    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in COMMANDS:
        print(__doc__.strip().split("\n\n")[0] + "\n\ncommands:")
        for name, (_, doc) in COMMANDS.items():
            print(f"  {name:14s} {doc}")
        return 0 if argv and argv[0] in ("-h", "--help") else (2 if argv else 0)
    mod = importlib.import_module(COMMANDS[argv[0]][0])
    mod.main(argv[1:])
    return 0


if __name__ == "__main__":
    sys.exit(main())
