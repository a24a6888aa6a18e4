"""Command-line entry point; the tool lives in micro_engram/tools/extract.py (run with --help)."""
from micro_engram.tools.extract import main

if __name__ == "__main__":
    main()
