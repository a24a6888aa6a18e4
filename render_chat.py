"""Command-line entry point; the tool lives in micro_engram/tools/render_chat.py (run with --help)."""
from micro_engram.tools.render_chat import main

if __name__ == "__main__":
    main()
