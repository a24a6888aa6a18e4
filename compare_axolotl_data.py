"""Command-line entry point; the tool lives in micro_engram/tools/compare_axolotl.py (run with --help)."""
from micro_engram.tools.compare_axolotl import main

if __name__ == "__main__":
    main()
