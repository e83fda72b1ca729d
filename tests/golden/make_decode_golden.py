"""Generate the seeded config-3 decode fixtures with the CPU oracle (no GPU, no reference code).

    python tests/golden/make_decode_golden.py bf16 [--steps 256]
    python tests/golden/make_decode_golden.py q8 [--steps 48]

Both build the BASELINE config-3 model (40 layers, 64 experts top-8, hidden 2048, GQA 32/4 x
128, dense layer 0 with intermediate 8192, vocabulary 100,352, RoPE theta 1e6, seed 1) on the
CPU from ``synth.decoder_tensors`` — the counter-based generator that gives the GPU build the
same bits — quantized by the oracle's quantizer (bit-exact with the library's GPU quantizer),
and run ``oracle/model_ref.py``, the restatement of laguna_mlx/laguna.py:75-206 that the
replay harness's greedy loop (laguna_mlx/dflash.py:102-112) and bench_kv.decode_at_ctx
(scripts/bench_kv.py:55-72) drive.

* ``bf16`` -> decode_config3_bf16.npz: the 8,192-token uniform-random prompt of seed 1
  (torch CPU generator, what bench.py's config-3 workload uses), bf16 KV cache, then
  greedy decoding. Stores per step the chosen token, the top-2 margin and the 8 largest
  logits with their ids, and the same for the prefill's last position.
* ``q8`` -> decode_config3_q8_82k.npz: the headline context. The CPU cannot prefill 82,671
  tokens through 40 layers (quadratic attention: petaflops), so every layer's cache starts
  from ``synth.kv_rows`` (hash N(0,1) K/V rows quantized 8-bit g64) holding 82,671 rows;
  the decode then starts at position 82,671 from token ``START_TOKEN`` with the 8-bit cache
  semantics of DequantKVCache(fused_decode=True) (laguna_mlx/cache.py:89-106).

The 256-step bf16 run takes about an hour on 8 cores; the q8 run with 48 steps about 20
minutes. The fixtures are small (tokens and logits only) and committed.
"""
import argparse
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
ROOT = OUT.parent.parent
sys.path.insert(0, str(ROOT))

from lagunalab_b200 import synth  # noqa: E402  (argument and tensor generators only)
from oracle import attn_ref, mlx_quant, model_ref  # noqa: E402

SEED = 1
PREFILL = 8192
Q8_CONTEXT = 82671
START_TOKEN = 4242
TOP = 8


def quantize(t, bits, threads=8):
    """The oracle's quantizer over row blocks in threads -> (int32 words, bf16 scales,
    bf16 biases) torch tensors."""
    x = t.reshape(-1, t.shape[-1]).numpy()
    blocks = np.array_split(np.arange(x.shape[0]), threads)
    with ThreadPoolExecutor(threads) as ex:
        parts = list(ex.map(lambda r: attn_ref.quantize_rows(x[r[0]:r[-1] + 1], 64, bits),
                            [b for b in blocks if len(b)]))
    q = np.concatenate([p[0] for p in parts]).reshape(*t.shape[:-1], -1)
    s = np.concatenate([p[1] for p in parts]).reshape(*t.shape[:-1], -1)
    b = np.concatenate([p[2] for p in parts]).reshape(*t.shape[:-1], -1)
    return (torch.from_numpy(q.view(np.int32)),
            torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))


def build():
    args = synth.decoder_args()
    t0 = time.time()
    W = model_ref.weights_from_named(synth.decoder_tensors(args, seed=SEED, device="cpu"),
                                     args.num_hidden_layers, quantize)
    print(f"weights built in {time.time() - t0:.0f} s", flush=True)
    return args, W, synth.oracle_args(args)


def _record(logits, toks, gaps, tvals, tids):
    last = logits[-1]
    top = torch.topk(last, TOP)
    toks.append(int(torch.argmax(last)))
    gaps.append(float(top.values[0] - top.values[1]))
    tvals.append(top.values.numpy().astype(np.float32))
    tids.append(top.indices.numpy().astype(np.int32))


def _save(path, toks, gaps, tvals, tids, **meta):
    np.savez_compressed(path, tokens=np.array(toks, np.int32), gaps=np.array(gaps, np.float32),
                        top_vals=np.stack(tvals), top_ids=np.stack(tids),
                        **{k: np.array(v) for k, v in meta.items()})


def run_bf16(steps):
    args, W, oa = build()
    prompt = torch.randint(0, args.vocab_size, (PREFILL,),
                           generator=torch.Generator().manual_seed(SEED))
    cache = model_ref.Cache(args.num_hidden_layers, None, capacity=PREFILL + steps + 1)
    t0 = time.time()
    logits = model_ref.forward(W, oa, prompt, cache, last_only=True)
    print(f"prefill {PREFILL} tokens in {time.time() - t0:.0f} s", flush=True)
    toks, gaps, tvals, tids = [], [], [], []
    path = OUT / "decode_config3_bf16.npz"
    for i in range(steps):
        _record(logits, toks, gaps, tvals, tids)
        if i + 1 < steps:
            t1 = time.time()
            logits = model_ref.forward(W, oa, [toks[-1]], cache)
            print(f"step {i + 1}: token {toks[-1]} margin {gaps[-1]:.4f} "
                  f"({time.time() - t1:.1f} s)", flush=True)
        if (i + 1) % 16 == 0 or i + 1 == steps:
            _save(path, toks, gaps, tvals, tids, seed=SEED, prefill=PREFILL, kv="bf16")
    print(f"wrote {path} ({len(toks)} steps)")


def run_q8(steps):
    args, W, oa = build()
    L = args.num_hidden_layers
    cache = model_ref.Cache(L, 8, capacity=Q8_CONTEXT + steps + 1)
    t0 = time.time()
    for i in range(L):
        k, v = synth.kv_rows(i, Q8_CONTEXT, args.num_key_value_heads, args.head_dim, seed=SEED,
                             device="cpu")
        rows = []
        for x in (k, v):
            q, s, b = quantize(x.float(), 8)
            rows.append(torch.from_numpy(mlx_quant.dequantize(
                q.numpy().view(np.uint32), s.view(torch.int16).numpy().view(np.uint16),
                b.view(torch.int16).numpy().view(np.uint16), 64, 8)))
        cache.preload(i, rows[0], rows[1])
    cache.offset = Q8_CONTEXT
    print(f"cache state built in {time.time() - t0:.0f} s", flush=True)
    toks, gaps, tvals, tids = [], [], [], []
    path = OUT / "decode_config3_q8_82k.npz"
    nxt = START_TOKEN
    for i in range(steps):
        t1 = time.time()
        logits = model_ref.forward(W, oa, [nxt], cache)
        _record(logits, toks, gaps, tvals, tids)
        nxt = toks[-1]
        print(f"step {i}: token {nxt} margin {gaps[-1]:.4f} ({time.time() - t1:.1f} s)",
              flush=True)
        if (i + 1) % 8 == 0 or i + 1 == steps:
            _save(path, toks, gaps, tvals, tids, seed=SEED, context=Q8_CONTEXT,
                  start_token=START_TOKEN, kv="q8")
    print(f"wrote {path} ({len(toks)} steps)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["bf16", "q8"])
    ap.add_argument("--steps", type=int, default=None)
    a = ap.parse_args()
    torch.set_num_threads(8)
    if a.case == "bf16":
        run_bf16(a.steps or 256)
    else:
        run_q8(a.steps or 48)


if __name__ == "__main__":
    main()
