"""Generate tests/golden/*.npz from the reference implementation itself.

Run in a container where the reference tree exists (its CPU sources are
compiled into oracle/_ref/libsa_ref.so by `make -C oracle`):

    python tests/golden/make_golden.py

Each fixture stores the generating seed, a digest of the regenerated inputs
(so a test can tell that it rebuilt the same inputs) and the reference's
outputs.  The reference ships no golden vectors of its own; these are the
outputs of its own functions on seeded inputs:
  * attention/src naive_attention_serial, streaming_attention_serial and
    streaming_attention_omp (unscaled, block 64);
  * per-head streaming_attention_omp for GQA decode (q pre-scaled by 1/sqrt(d));
  * tensor_cpp ops::self_attention_streaming_blockwise and ops::self_attention
    (causal) for prefill;
  * tensor_cpp qwen3_forward and qwen3_forward_with_cache (STANDARD) for a
    small random-init Qwen3.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle.oracle import Qwen3Cfg, Reference, bf16_round, make_qwen3_weights  # noqa: E402
import _inputs as I  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# small Qwen3-shaped model for the forward fixtures (real head_dim / GQA ratio)
TINY = dict(vocab=2048, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=768,
            eps=1e-6, theta=1e6)
TINY_SEED = 1234
TINY_PROMPT_SEED = 99


def main() -> None:
    R = Reference()
    # ---- single-query attention.h kernels
    rec = {}
    for i, (T, d) in enumerate(I.SINGLE_CASES):
        seed = 100 + i
        q, k, v = I.single_query(T, d, seed)
        rec[f"c{i}_meta"] = np.array([T, d, seed, 64], np.int64)
        rec[f"c{i}_digest"] = np.array(I.digest(q, k, v))
        rec[f"c{i}_naive"] = R.naive_serial(q, k, v)
        rec[f"c{i}_streaming"] = R.streaming_serial(q, k, v, 64)
        rec[f"c{i}_omp4"] = R.streaming_omp(q, k, v, 64, 4)
    np.savez_compressed(os.path.join(OUT, "single_query.npz"), **rec)

    # ---- GQA decode (fp32 and bf16-rounded inputs)
    rec = {}
    for i, (hq, hkv, T, d) in enumerate(I.GQA_CASES):
        seed = 200 + i
        q, k, v = I.gqa(hq, hkv, T, d, seed)
        s = 1.0 / np.sqrt(d)
        rec[f"c{i}_meta"] = np.array([hq, hkv, T, d, seed], np.int64)
        rec[f"c{i}_digest"] = np.array(I.digest(q, k, v))
        rec[f"c{i}_out"] = R.gqa_decode_omp(q, k, v, 64, 4, s)
        qb, kb, vb = bf16_round(q), bf16_round(k), bf16_round(v)
        rec[f"c{i}_out_bf16in"] = R.gqa_decode_omp(qb, kb, vb, 64, 4, s)
    np.savez_compressed(os.path.join(OUT, "gqa_decode.npz"), **rec)

    # ---- causal prefill
    rec = {}
    for i, (S, hq, hkv, d) in enumerate(I.PREFILL_CASES):
        seed = 300 + i
        q, k, v = I.prefill(S, hq, hkv, d, seed)
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
        s = 1.0 / np.sqrt(d)
        rec[f"c{i}_meta"] = np.array([S, hq, hkv, d, seed], np.int64)
        rec[f"c{i}_digest"] = np.array(I.digest(q, k, v))
        bw = R.causal_prefill(q, k, v, s, 32, 64, standard=False)
        st = R.causal_prefill(q, k, v, s, standard=True)
        rec[f"c{i}_blockwise"] = bw
        # the masked standard path agrees with the block-wise one; keep only the gap
        rec[f"c{i}_standard_gap"] = np.array(np.abs(bw - st).max(), np.float32)
    np.savez_compressed(os.path.join(OUT, "causal_prefill.npz"), **rec)

    # ---- Qwen3 tiny forward + cached greedy decode
    cfg = Qwen3Cfg(**TINY)
    w = make_qwen3_weights(cfg, TINY_SEED)
    ids = I.rng(TINY_PROMPT_SEED).integers(0, cfg.vocab, 24).astype(np.int64)
    m = R.qwen3(cfg, w)
    logits = m.forward(ids)
    kv = m.new_cache(64)
    cached = m.forward_cached(kv, ids)
    toks = []
    nxt = int(np.argmax(cached[-1]))
    steps = []
    for _ in range(6):
        toks.append(nxt)
        lg = m.forward_cached(kv, np.array([nxt], np.int64))
        steps.append(lg[0])
        nxt = int(np.argmax(lg[0]))
    m.free_cache(kv)
    np.savez_compressed(
        os.path.join(OUT, "qwen3_tiny.npz"),
        cfg=np.array([TINY[k] for k in ("vocab", "hidden", "n_layers", "hq", "hkv", "head_dim",
                                         "inter")], np.int64),
        seeds=np.array([TINY_SEED, TINY_PROMPT_SEED], np.int64),
        weights_digest=np.array(I.digest(w["embed"], w["layers"])),
        ids=ids, logits_last4=logits[-4:], greedy_tokens=np.array(toks, np.int64),
        decode_logits=np.stack(steps))
    print("fixtures written to", OUT)


if __name__ == "__main__":
    main()
