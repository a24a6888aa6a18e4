"""Command-line tools around trained engrams: token merging (build_canon), model assembly
(assemble, extract), checkpoint inspection (engram_stats), ablations (zero_order), data
statistics (data_stats, compare_axolotl), chat rendering and held-out scoring against a
vLLM server (render_chat, eval_logprob, token_diff), and HF inference / an OpenAI-style
server (infer, serve). Each module runs as `python -m micro_engram.tools.<name>`; the
same-named scripts at the repository root call them."""
