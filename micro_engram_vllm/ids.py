"""Token histories for the serving engram: for every token a vLLM step runs, that token and
the ones before it in its request (reference: micro_engram_vllm/ids.py:10-70).

Rule, per token t of request r at position p and history slot i:
    q = p - i;  q < 0 -> -1 (before the request);  q >= first position of r's chunk in this
    step -> input_ids[t - i] (same chunk);  else -> all_token_ids[idx_mapping[r], q] (earlier
    chunks, earlier decode steps, prefix-cache hits, restored tokens).
Rows past num_tokens (CUDA-graph padding) are -1. On CUDA this is one sm_100a kernel
(`micro_engram_b200::fill_ids`) that reads no value back to the host, so it can run before
every step and under graph replay; on CPU the same rule runs as torch ops.
"""
import torch


def fill_engram_ids(out, input_ids, positions, idx_mapping, query_start_loc, all_token_ids, num_reqs,
                    num_tokens, num_tokens_padded):
    """Write out[:num_tokens_padded] ([max_tokens, max_order] int32) in place."""
    if out.is_cuda:
        from micro_engram_fork_b200.ops.registry import fill_ids

        fill_ids(out, input_ids, positions, idx_mapping, query_start_loc, all_token_ids, int(num_reqs),
                 int(num_tokens), int(num_tokens_padded))
        return
    max_order = out.shape[1]
    if num_tokens > 0:
        qsl = query_start_loc[: num_reqs + 1].long()
        tok = torch.arange(num_tokens)
        req = torch.searchsorted(qsl[1:], tok, right=True).clamp(max=num_reqs - 1)
        pos = positions[:num_tokens].long()
        ids = input_ids[:num_tokens].long()
        start = pos[qsl[:-1].clamp(max=num_tokens - 1)][req]
        slot = idx_mapping[:num_reqs].long()[req]
        i = torch.arange(max_order)
        q = pos[:, None] - i[None, :]
        chunk = ids[(tok[:, None] - i[None, :]).clamp(min=0)]
        hist = all_token_ids[slot[:, None], q.clamp(min=0)].long()
        val = torch.where(q >= start[:, None], chunk, hist)
        out[:num_tokens] = torch.where(q >= 0, val, torch.full_like(val, -1)).to(out.dtype)
    if num_tokens_padded > num_tokens:
        out[num_tokens:num_tokens_padded] = -1


def mask_media(ids, media_ids):
    """Media placeholder tokens get no engram and count as missing history.

    Returns (ids with every media id replaced by -1, keep [n] bool = token itself is not media)."""
    is_media = torch.isin(ids, media_ids.to(ids.dtype))
    return ids.masked_fill(is_media, -1), ~is_media[:, 0]
