"""Command-line entry point; the tool lives in micro_engram/tools/token_diff.py (run with --help)."""
from micro_engram.tools.token_diff import main

if __name__ == "__main__":
    main()
