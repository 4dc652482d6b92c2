"""Helpers shared by the tests: golden fixtures and case decoding."""

import json
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
_CACHE = {}


def golden(name):
    if name not in _CACHE:
        _CACHE[name] = np.load(GOLDEN / f"{name}.npz")
    return _CACHE[name]


def jload(arr):
    return json.loads(bytes(np.asarray(arr, np.uint8)).decode())


def case_names(kind):
    g = golden({"mask": "masks", "seg": "segmented", "tiled": "tiled", "num": "numerics"}[kind])
    return jload(g[f"{kind}_case_names"])


def mask_case(name):
    g = golden("masks")
    meta = jload(g[f"{name}/meta"])
    c = dict(meta)
    c["labels"] = g[f"{name}/labels"]
    c["active"] = g[f"{name}/active"] if f"{name}/active" in g else None
    if meta["mode"] == "membership":
        c["membership"] = g[f"{name}/membership"]
        c["global_only"] = g[f"{name}/global_only"]
    else:
        c["membership"] = None
        c["global_only"] = None
    S = meta["S"]
    c["dense"] = np.unpackbits(g[f"{name}/dense_bits"])[: S * S].reshape(S, S).astype(bool)
    for k in ("kv_num_blocks", "kv_indices", "full_kv_num_blocks", "full_kv_indices"):
        c[k] = g[f"{name}/{k}"]
    return c


def mask_kwargs(c):
    """Keyword arguments for the oracle / product mask builders."""
    return dict(labels=None if c["membership"] is not None else c["labels"],
                active=c["active"], direct=c["direct"], membership=c["membership"],
                global_only=c["global_only"], no_local=c["no_local"])


def seg_case(name):
    g = golden("segmented")
    meta = jload(g[f"{name}/meta"])
    out = {k: g[f"{name}/{k}"] for k in ("prog_qbase", "prog_nq", "prog_seg", "kv_index",
                                           "kv_count", "logical_pairs")}
    for k in ("q_index", "k_index", "cu_q", "cu_k", "scalars"):
        key = f"{name}/plan_{k}"
        if key in g:
            out[f"plan_{k}"] = g[key]
    return meta, out


def seg_kwargs(meta):
    to_t = lambda x: tuple(tuple(r) for r in x)  # noqa: E731
    return dict(P=meta["P"], N=meta["N"], L=meta["L"], KL=meta["KL"], KG=meta["KG"],
                n_frames=meta["n_frames"], n_block=meta["n_block"],
                local_attn=meta["local_attn"], agent=to_t(meta["agent"]),
                local=to_t(meta["local"]), glob=tuple(meta["glob"]),
                local_active=to_t(meta["local_active"]),
                labels=None if meta["labels"] is None else to_t(meta["labels"]),
                q_active=to_t(meta["q_active"]), direct=meta["direct"],
                membership=meta["membership"], global_only=meta["global_only"],
                no_local=meta["no_local"])


def tiled_case(name):
    g = golden("tiled")
    meta = jload(g[f"{name}/meta"])
    lays = []
    for i in range(int(g[f"{name}/n_layouts"])):
        d = {k: g[f"{name}/{i}/{k}"] for k in ("prog_qbase", "prog_nq", "prog_seg", "kv_index",
                                                "kv_count", "kv_valid", "slots")}
        lays.append(d)
    return meta, lays


def bf16_bits_to_f32(a):
    a = np.asarray(a, np.uint16).astype(np.uint32) << 16
    return a.view(np.float32)


def num_case(name):
    g = golden("numerics")
    meta = jload(g[f"{name}/meta"])
    d = {"meta": meta}
    for k in ("qx", "kx", "v", "cam", "wcq", "wck", "nqw", "nkw"):
        d[k] = bf16_bits_to_f32(g[f"{name}/{k}"])
        d[k + "_bits"] = g[f"{name}/{k}"]
    for k in ("freqs", "cam12", "labels", "roped_q", "roped_k", "out", "mask_popcount"):
        d[k] = g[f"{name}/{k}"]
    if f"{name}/membership" in g:
        d["membership"] = g[f"{name}/membership"]
        d["global_only"] = g[f"{name}/global_only"]
    return d
