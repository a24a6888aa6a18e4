"""Command-line entry point; the tool lives in micro_engram/tools/engram_stats.py (run with --help)."""
from micro_engram.tools.engram_stats import main

if __name__ == "__main__":
    main()
