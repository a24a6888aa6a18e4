"""Command-line entry point; the tool lives in micro_engram/tools/zero_order.py (run with --help)."""
from micro_engram.tools.zero_order import main

if __name__ == "__main__":
    main()
