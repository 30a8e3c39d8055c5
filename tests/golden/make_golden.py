"""Generate the golden fixtures in this directory from the reference itself.

Run in a container that has the reference checkout (read-only); its path
is required in ``$Q6W_REFERENCE``:

    Q6W_REFERENCE=<checkout> python tests/golden/make_golden.py
    Q6W_REFERENCE=<checkout> python tests/golden/make_golden.py --copy-shipped

``--copy-shipped`` only copies the shipped QAT artifact (binary + manifest,
1.1 MB, public) into ``tests/golden/shipped/``, which git ignores: the GPU
test of the shipped request finds it there on a machine without the
checkout, and it is never committed.

It imports the reference's own ``quantization/q6w_format.py`` and
``benchmarks/torch_benchmark.py`` and records what they produce:

* ``codec.json``   -- packed bytes from the reference packer and the codes its
  unpacker returns (including hand-made bytes holding the code 0x20 = -32,
  which the reference decodes but never packs), plus ``quantize_rows``
  outputs on seeded matrices with an all-zero row and exact .5 ties;
* ``tiny_request.json`` -- the tiny synthetic model (dim 128, 5 layers, 8 q
  heads, 4 kv heads, hidden 384, vocab 4096, context 256; weights N(0, 0.02)
  from seed 1234, written by q6w_b200.format.write_synthetic and loaded by
  the reference's ``load_dequantized_state``): a 20-token prompt drawn
  U[3, 4095] from seed 7, 128 greedy tokens from the reference ``generate``,
  the same request with a stop id and ``min_new_tokens`` through the
  ``prepare_e2e`` loop, per-step top-1/top-2 margins, and the SHA-256 of the
  binary so the writer + seed are pinned;
* ``tiny_logits.npz`` -- reference logits of the last prompt step and the
  first decode steps;
* ``shipped_request.json`` -- the shipped QAT artifact on the standard
  story-opening request (prompt ids from the shipped tokenizer), 128 greedy
  tokens with min_new_tokens 4 and stop ids {BOS, EOS}.  The artifact itself
  is not copied here.

``--sampling`` writes only the two fixtures below (the others stay as recorded):

* ``sampling.json`` -- the reference's ``generate`` at temperature > 0 and
  with its logit processors (repetition penalty, n-gram blocking, stop-id
  masking and bias) on the tiny synthetic model and the golden prompt, six
  settings, 64 tokens each;
* ``fp16_kv.json`` / ``fp16_kv_logits.npz`` -- the reference's FP16-KV
  wrapper (quantization/compare_kv_cache.py) on the same request: 128 greedy
  tokens and the logits of the last prompt step and four decode steps.
"""

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("Q6W_REFERENCE"):
    sys.exit("set Q6W_REFERENCE to the reference checkout")
REF = Path(os.environ["Q6W_REFERENCE"])
sys.path.insert(0, str(REPO / "tinyllm-pynq-z2_b200"))
sys.path.insert(0, str(REF / "quantization"))
sys.path.insert(0, str(REF / "benchmarks"))

import q6w_format as ref_fmt  # noqa: E402
import torch_benchmark as ref_tb  # noqa: E402
from q6w_b200 import format as fmt  # noqa: E402

DEFAULTS = {"hidden_dim": None, "multiple_of": 256, "norm_eps": 1e-5, "n_kv_heads": None, "max_seq_len": 2048,
            "dropout": 0.0}
TINY_SEED = 1234
PROMPT_SEED = 7


def codec_vectors():
    rng = np.random.default_rng(20261201)
    out = {"pack": [], "unpack_only": [], "quantize": []}
    for rows, cols in ((1, 4), (3, 16), (4, 128), (2, 352)):
        q = rng.integers(-31, 32, size=(rows, cols))
        packed = ref_fmt.pack_signed_int6(q)
        back = ref_fmt.unpack_signed_int6(packed, rows, cols)
        out["pack"].append({"rows": rows, "cols": cols, "codes": q.tolist(), "packed_hex": packed.hex(),
                            "unpacked": back.tolist()})
    # every 6-bit pattern, 0x20 (-32) included, from raw bytes
    fields = np.arange(64, dtype=np.int64).reshape(16, 4)
    word = fields[:, 0] | (fields[:, 1] << 6) | (fields[:, 2] << 12) | (fields[:, 3] << 18)
    raw = np.stack([word & 255, (word >> 8) & 255, (word >> 16) & 255], axis=1).astype(np.uint8).tobytes()
    out["unpack_only"].append({"rows": 1, "cols": 64, "packed_hex": raw.hex(),
                               "unpacked": ref_fmt.unpack_signed_int6(raw, 1, 64).tolist()})
    raw2 = bytes(rng.integers(0, 256, size=3 * 8 * 12, dtype=np.uint8))
    out["unpack_only"].append({"rows": 8, "cols": 48, "packed_hex": raw2.hex(),
                               "unpacked": ref_fmt.unpack_signed_int6(raw2, 8, 48).tolist()})
    g = torch.Generator().manual_seed(99)
    w = torch.empty(6, 32).normal_(0, 0.02, generator=g)
    w[2] = 0.0
    w[3] = torch.tensor([0.5, -1.5, 2.5, 31.0] * 8) / 31.0 * 0.1  # exact-ish ties after scaling
    w[4, :4] = torch.tensor([1.0, -1.0, 0.5, -0.5])
    q, s, stats = ref_fmt.quantize_rows(w)
    out["quantize"].append({"weights": w.tolist(), "q": q.tolist(), "scales": s.astype(np.float32).tolist(),
                            "stats": stats})
    return out


def load_reference_model(bin_path, manifest_path, max_seq_len=None):
    manifest = json.loads(Path(manifest_path).read_text())
    shapes = fmt._model_shapes(manifest["model_args"])
    template = {k: torch.zeros(v) for k, v in shapes.items()}
    template["output.weight"] = template["tok_embeddings.weight"]
    state, manifest = ref_fmt.load_dequantized_state(bin_path, manifest_path, template)
    args = SimpleNamespace(**{**DEFAULTS, **manifest["model_args"]})
    if max_seq_len:
        args.max_seq_len = max_seq_len
    model = ref_tb.CachedTransformer(args).eval()
    model.load_state_dict(state, strict=True)
    return model, manifest


def greedy_with_stops(model, prompt, new_tokens, stop_ids, min_new):
    """scripts/prepare_e2e.py:120-143, verbatim in behaviour."""
    k, v = model.new_cache(torch.device("cpu"))
    rows, sampled, generated, margins = [], [], [], []
    stopped_on = None
    with torch.inference_mode():
        for pos, tok in enumerate(prompt):
            logits = model.step(tok, pos, k, v)
        for index in range(new_tokens):
            rows.append(logits.clone())
            scores = logits.clone()
            if index < min_new:
                for t in stop_ids:
                    scores[t] = -float("inf")
            t = int(torch.argmax(scores).item())
            top2 = torch.topk(scores, 2).values
            margins.append(float(top2[0] - top2[1]))
            sampled.append(t)
            if index >= min_new and t in stop_ids:
                stopped_on = t
                break
            generated.append(t)
            if index + 1 < new_tokens:
                logits = model.step(t, len(prompt) + index, k, v)
    return {"sampled": sampled, "generated": generated, "stopped_on": stopped_on, "margins": margins,
            "logits": torch.stack(rows)}


def tiny_request(tmp):
    b, m = tmp / "tiny.bin", tmp / "tiny.json"
    fmt.write_synthetic(fmt.TINY_ARGS, TINY_SEED, b, m)
    sha = hashlib.sha256(b.read_bytes()).hexdigest()
    model, manifest = load_reference_model(b, m)
    prompt = torch.randint(3, 4096, (20,), generator=torch.Generator().manual_seed(PROMPT_SEED)).tolist()
    with torch.inference_mode():
        gen, _, _, stopped, reason = ref_tb.generate(model, prompt, 128, torch.device("cpu"))
    plain = greedy_with_stops(model, prompt, 128, [], 0)
    assert plain["generated"] == gen
    # a stop id the model really emits, so masking and stopping both engage
    distinct = [t for t in dict.fromkeys(gen)]
    stop_id = distinct[1] if len(distinct) > 1 else distinct[0]
    min_new = 3
    stop_run = greedy_with_stops(model, prompt, 128, [stop_id], min_new)
    logits = {"prompt_last": plain["logits"][0].numpy(), "decode_1_4": plain["logits"][1:5].numpy(),
              "stop_run_first": stop_run["logits"][0].numpy()}
    doc = {
        "model_args": manifest["model_args"], "seed": TINY_SEED, "binary_sha256": sha,
        "binary_bytes": b.stat().st_size, "prompt_seed": PROMPT_SEED, "prompt": prompt, "new_tokens": 128,
        "generated": gen, "stopped": stopped, "margins": plain["margins"],
        "stop_case": {"stop_ids": [stop_id], "min_new_tokens": min_new, "sampled": stop_run["sampled"],
                      "generated": stop_run["generated"], "stopped_on": stop_run["stopped_on"]},
        "torch": torch.__version__,
    }
    return doc, logits


def shipped_request():
    art = REF / "quantization" / "artifacts"
    b, m = art / "tinyllamas_zh_story_q6w_qat_lr1e6.bin", art / "tinyllamas_zh_story_q6w_qat_lr1e6.json"
    manifest = json.loads(m.read_text())
    model, manifest = load_reference_model(b, m, manifest["model_args"]["max_seq_len"])
    from sentencepiece import SentencePieceProcessor

    sp = SentencePieceProcessor(model_file=str(REF / "tok4096.model"))
    text = "故事开头：{}\n续写：".format("从前，有一只叫小白的兔子。")
    prompt = [int(sp.bos_id())] + [int(t) for t in sp.encode(text)]
    stop_ids = sorted({int(sp.bos_id()), int(sp.eos_id())})
    run = greedy_with_stops(model, prompt, 128, stop_ids, 4)
    return {"binary_file": b.name, "binary_sha256": manifest["binary_sha256"], "model_args": manifest["model_args"],
            "prompt": prompt, "new_tokens": 128, "min_new_tokens": 4, "stop_ids": stop_ids,
            "sampled": run["sampled"], "generated": run["generated"], "stopped_on": run["stopped_on"],
            "margins": run["margins"], "torch": torch.__version__}


SAMPLING_CASES = [
    {"temperature": 0.8, "top_p": 0.9, "seed": 1},
    {"temperature": 1.0, "top_p": 1.0, "seed": 7},
    {"temperature": 0.7, "top_p": 0.95, "seed": 3, "repetition_penalty": 1.3, "no_repeat_ngram_size": 3},
    {"temperature": 0.9, "top_p": 0.9, "seed": 11, "min_new_tokens": 4, "stop_token_bias": 8.0,
     "stop_token_bias_after": 8, "stop": True},
    {"temperature": 0.0, "top_p": 0.9, "seed": 1, "repetition_penalty": 1.2, "no_repeat_ngram_size": 2},
    {"temperature": 1.2, "top_p": 0.5, "seed": 42, "no_repeat_ngram_size": 1},
]


def sampling_requests(tmp):
    """The reference's own ``generate`` at temperature > 0 and with its logit
    processors, on the tiny synthetic model and the golden 20-token prompt."""
    b, m = tmp / "tiny.bin", tmp / "tiny.json"
    fmt.write_synthetic(fmt.TINY_ARGS, TINY_SEED, b, m)
    model, _ = load_reference_model(b, m)
    prompt = torch.randint(3, 4096, (20,), generator=torch.Generator().manual_seed(PROMPT_SEED)).tolist()
    cases = []
    stop_id = None
    for case in SAMPLING_CASES:
        kw = {k: v for k, v in case.items() if k != "stop"}
        if case.get("stop"):
            kw["stop_token"] = {stop_id}
        with torch.inference_mode():
            gen, _, _, stopped, reason = ref_tb.generate(model, prompt, 64, torch.device("cpu"), **kw)
        if stop_id is None:
            stop_id = gen[12]  # a token the model samples, for the stop case
        cases.append({"kwargs": {k: (sorted(v) if isinstance(v, set) else v) for k, v in kw.items()},
                      "new_tokens": 64, "generated": gen, "stopped": stopped, "stop_reason": reason})
    return {"seed": TINY_SEED, "prompt": prompt, "cases": cases, "torch": torch.__version__}


def fp16_kv_request(tmp):
    """The reference's FP16-KV wrapper (quantization/compare_kv_cache.py:15-72)
    on the tiny synthetic model: the golden prompt + 128 greedy tokens, and
    the logits of the last prompt step and the first decode steps."""
    sys.path.insert(0, str(REF / "quantization"))
    import compare_kv_cache as ref_kv

    b, m = tmp / "tiny16.bin", tmp / "tiny16.json"
    fmt.write_synthetic(fmt.TINY_ARGS, TINY_SEED, b, m)
    model, _ = load_reference_model(b, m)
    fp16 = ref_kv.FP16KVTransformer(model)
    prompt = torch.randint(3, 4096, (20,), generator=torch.Generator().manual_seed(PROMPT_SEED)).tolist()
    with torch.inference_mode():
        gen, _, _, _, _ = ref_tb.generate(fp16, prompt, 128, torch.device("cpu"))
        k, v = fp16.new_cache(torch.device("cpu"))
        rows = []
        for pos, tok in enumerate(prompt + gen[:4]):
            lg = fp16.step(tok, pos, k, v)
            if pos >= len(prompt) - 1:
                rows.append(lg.clone())
    return {"prompt": prompt, "generated": gen}, torch.stack(rows).numpy()


def forward_all_request(tmp):
    """The reference's non-cached forward with targets (training/model.py
    Transformer.forward, :249-269) on the tiny synthetic model: a [2, 40]
    token batch whose targets ignore (-1) a few positions; the loss and the
    logits of every 5th position."""
    sys.path.insert(0, str(REF / "training"))
    import model as ref_train

    b, m = tmp / "tinyf.bin", tmp / "tinyf.json"
    fmt.write_synthetic(fmt.TINY_ARGS, TINY_SEED, b, m)
    manifest = json.loads(m.read_text())
    margs = {**DEFAULTS, **manifest["model_args"]}
    args = ref_train.ModelArgs(**{k: margs[k] for k in ("dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
                                                         "hidden_dim", "multiple_of", "norm_eps", "max_seq_len",
                                                         "dropout")})
    model = ref_train.Transformer(args).eval()
    template = {k: v.detach().clone() for k, v in model.state_dict().items()}
    state, _ = ref_fmt.load_dequantized_state(b, m, template)
    model.load_state_dict(state, strict=True)
    g = torch.Generator().manual_seed(41)
    tokens = torch.randint(3, 4096, (2, 40), generator=g)
    targets = torch.roll(tokens, -1, dims=1)
    targets[:, -1] = -1
    targets[1, :7] = -1
    with torch.inference_mode():
        logits = model(tokens, targets)
        loss = float(model.last_loss)
    return ({"tokens": tokens.tolist(), "targets": targets.tolist(), "loss": loss, "rows_every": 5,
             "torch": torch.__version__}, logits[:, ::5].numpy())


SHIPPED = "tinyllamas_zh_story_q6w_qat_lr1e6"


def copy_shipped():
    import shutil

    dst = HERE / "shipped"
    dst.mkdir(exist_ok=True)
    for ext in (".bin", ".json"):
        shutil.copyfile(REF / "quantization" / "artifacts" / (SHIPPED + ext), dst / (SHIPPED + ext))
    print("shipped artifact copied to", dst)


def main():
    if "--copy-shipped" in sys.argv:
        copy_shipped()
        return
    torch.set_num_threads(1)
    if "--sampling" in sys.argv:  # only the sampling and FP16-KV fixtures (the others stay as recorded)
        with tempfile.TemporaryDirectory() as d:
            (HERE / "sampling.json").write_text(json.dumps(sampling_requests(Path(d)), indent=1) + "\n")
            doc, rows = fp16_kv_request(Path(d))
        (HERE / "fp16_kv.json").write_text(json.dumps(doc, indent=1) + "\n")
        np.savez_compressed(HERE / "fp16_kv_logits.npz", rows=rows)
        print("sampling and FP16-KV fixtures written to", HERE)
        return
    if "--forward" in sys.argv:  # only the non-cached forward fixture
        with tempfile.TemporaryDirectory() as d:
            doc, rows = forward_all_request(Path(d))
        (HERE / "forward_all.json").write_text(json.dumps(doc, indent=1) + "\n")
        np.savez_compressed(HERE / "forward_all_logits.npz", rows=rows)
        print("forward fixture written to", HERE)
        return
    (HERE / "codec.json").write_text(json.dumps(codec_vectors(), indent=1) + "\n")
    with tempfile.TemporaryDirectory() as d:
        doc, logits = tiny_request(Path(d))
    (HERE / "tiny_request.json").write_text(json.dumps(doc, indent=1) + "\n")
    np.savez_compressed(HERE / "tiny_logits.npz", **logits)
    (HERE / "shipped_request.json").write_text(json.dumps(shipped_request(), ensure_ascii=False, indent=1) + "\n")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
