"""Command-line entry point: add trained engram(s) to a Gemma 4 GGUF for the engram runtime
and the llama.cpp patch; the code is micro_engram/gguf_export.py (run with --help)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # the repository root

from micro_engram.gguf_export import main  # noqa: E402

if __name__ == "__main__":
    main()
