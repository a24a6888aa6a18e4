"""Command-line entry point; the tool lives in micro_engram/tools/build_canon.py (run with --help)."""
from micro_engram.tools.build_canon import main

if __name__ == "__main__":
    main()
