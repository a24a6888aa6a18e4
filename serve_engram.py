"""Command-line entry point; the tool lives in micro_engram/tools/serve.py (run with --help)."""
from micro_engram.tools.serve import main

if __name__ == "__main__":
    main()
