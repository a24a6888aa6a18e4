"""Command-line entry point; the tool lives in micro_engram/tools/eval_logprob.py (run with --help)."""
from micro_engram.tools.eval_logprob import main

if __name__ == "__main__":
    main()
