"""Tensor-parallel helpers around lmc_model_load_tp (one process per GPU).

shard_plan() restates the C runtime's shard geometry (lmc_b200/host/
lmc_model.c, load): rank r of N holds query heads [r H/N, (r+1) H/N) with
kv heads [r Hkv/N, ...), ffn rows [r F/N, ...) of gate / up (the same columns
of down), the attn_output columns of its heads, and lm_head rows
[r ceil(V/N), ...).  exchange_id() hands one NCCL group id from rank 0 to
every rank over an existing torch.distributed group (gloo or nccl).
"""


def shard_plan(cfg, rank, size):
    """cfg: object with n_heads, n_kv_heads, head_dim, ffn_dim, vocab_size."""
    if cfg.n_heads % size or cfg.n_kv_heads % size or cfg.ffn_dim % size:
        raise ValueError("heads, kv heads and ffn rows must divide by the group size")
    hl, hkvl, fl = cfg.n_heads // size, cfg.n_kv_heads // size, cfg.ffn_dim // size
    vr = -(-cfg.vocab_size // size)
    v0 = rank * vr
    return {"q_rows": (rank * hl * cfg.head_dim, hl * cfg.head_dim),
            "kv_rows": (rank * hkvl * cfg.head_dim, hkvl * cfg.head_dim),
            "ffn_rows": (rank * fl, fl),
            "o_cols": (rank * hl * cfg.head_dim, hl * cfg.head_dim),
            "down_cols": (rank * fl, fl),
            "vocab_rows": (v0, max(0, min(vr, cfg.vocab_size - v0)))}


def exchange_id(dist, make_id):
    """Rank 0 calls make_id() (a 128-byte NCCL id); every rank returns it."""
    obj = [make_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]
