#!/usr/bin/env python
"""End-to-end vLLM offline throughput with the B200 backend plugged in.

Workload: a Llama-3-8B-shaped decoder (32 layers, hidden 4096, 32/8 heads of 128,
intermediate 14336, vocab 128256, RMSNorm eps 1e-5, RoPE base 500000) with vLLM's dummy
weights (no checkpoint is available offline), 256 prompts of 512 uniform random token ids,
128 greedy tokens each (ignore_eos), FLASH_ATTN backend (``--attention-backend
FLASHINFER`` for vLLM's FlashInfer backend), eager mode.

    python bench_vllm.py --mode b200|native [--replicas N | --tp N]

``b200``: the vllm_nt plugin is discovered the way an installed plugin is (a
``vllm.general_plugins`` entry point on PYTHONPATH, so tensor-parallel workers load it
too) with every hooked op on the B200 kernels (configs/all-b200.yaml).  ``native``: no
plugin, vLLM's own CUDA ops.  ``--replicas N`` runs N independent single-GPU engines at
once (one per GPU, 256 prompts each) and reports the aggregate; ``--tp N`` runs one
engine with tensor parallelism N.  Each engine runs in a child process; it prints
``RESULT_JSON=`` with output tokens/s and, for in-process engines, the plugin's usage
summary.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "vllm-nt_b200"

LLAMA3_8B_SHAPE = {
    "architectures": ["LlamaForCausalLM"],
    "model_type": "llama",
    "hidden_size": 4096,
    "intermediate_size": 14336,
    "num_attention_heads": 32,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "num_hidden_layers": 32,
    "vocab_size": 128256,
    "rms_norm_eps": 1e-5,
    "rope_theta": 500000.0,
    "max_position_embeddings": 8192,
    "hidden_act": "silu",
    "tie_word_embeddings": False,
    "torch_dtype": "bfloat16",
    "bos_token_id": 128000,
    "eos_token_id": 128001,
    "attention_bias": False,
    "mlp_bias": False,
}


def write_model_dir(base: Path) -> Path:
    d = base / "llama3-8b-shape"
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(LLAMA3_8B_SHAPE, indent=1))
    return d


def write_plugin_dist(base: Path) -> Path:
    """A dist-info declaring the plugin's entry point, as `pip install` would create."""
    site = base / "plugin-site"
    dist = site / "vllm_nt-0.2.0.dist-info"
    dist.mkdir(parents=True, exist_ok=True)
    (dist / "METADATA").write_text("Metadata-Version: 2.1\nName: vllm-nt\nVersion: 0.2.0\n")
    (dist / "entry_points.txt").write_text("[vllm.general_plugins]\nvllm_nt = vllm_nt:register\n")
    return site


def _worker_usage(worker=None) -> dict:
    """Runs inside a vLLM worker process (collective_rpc): that rank's plugin counters."""
    from vllm_nt.oot import get_usage_summary

    s = get_usage_summary()
    return {"hit_ops": list(s["hit_ops"]),
            "operators": {k: {"hits": v["hits"], "failures": v["failures"], "fallbacks": v["fallbacks"],
                              "declined": v.get("declined", {})} for k, v in s["operators"].items()}}


def child(args) -> int:
    import numpy as np
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    llm = LLM(
        model=args.model_dir,
        skip_tokenizer_init=True,
        load_format="dummy",
        dtype="bfloat16",
        tensor_parallel_size=args.tp,
        enforce_eager=True,
        max_model_len=1024,
        max_num_seqs=256,
        gpu_memory_utilization=0.85,
        attention_backend=args.attention_backend,
        seed=0,
    )
    rng = np.random.default_rng(args.seed)
    prompts = [TokensPrompt(prompt_token_ids=rng.integers(0, 128256, 512).tolist()) for _ in range(args.prompts)]
    warm = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True, detokenize=False)
    llm.generate(prompts[:16], warm, use_tqdm=False)
    if args.sampling == "topkp":
        # one seed per request: vLLM then samples through TopKTopPSampler.forward_native (its
        # FlashInfer sampler takes no per-request generators), where the TopKTopP and
        # RandomSample hooks sit
        sp = [SamplingParams(temperature=0.8, top_k=50, top_p=0.9, seed=args.seed * 100003 + i,
                             max_tokens=args.output_len, min_tokens=args.output_len, ignore_eos=True,
                             detokenize=False) for i in range(len(prompts))]
    else:
        sp = SamplingParams(temperature=0.0, max_tokens=args.output_len, min_tokens=args.output_len,
                            ignore_eos=True, detokenize=False)
    t0 = time.perf_counter()
    outs = llm.generate(prompts, sp, use_tqdm=False)
    dt = time.perf_counter() - t0
    generated = sum(len(o.outputs[0].token_ids) for o in outs)
    result = {
        "mode": args.mode,
        "tp": args.tp,
        "sampling": args.sampling,
        "prompts": args.prompts,
        "output_tokens": generated,
        "seconds": dt,
        "output_tok_s": generated / dt,
        "total_tok_s": (generated + args.prompts * 512) / dt,
    }
    if args.mode == "b200":
        try:
            # tensor-parallel workers are other processes: ask each for its counters
            per_rank = llm.collective_rpc(_worker_usage) if args.tp > 1 else [_worker_usage()]
            s = {"hit_ops": sorted({op for r in per_rank for op in r["hit_ops"]}), "operators": {}}
            for r in per_rank:
                for k, v in r["operators"].items():
                    acc = s["operators"].setdefault(k, {"hits": 0, "failures": 0, "fallbacks": 0, "declined": {}})
                    for c in ("hits", "failures", "fallbacks"):
                        acc[c] += v[c]
                    for why, n in v["declined"].items():
                        acc["declined"][why] = acc["declined"].get(why, 0) + n
            ops_ = s["operators"]
            result["hit_ops"] = s["hit_ops"]
            result["hits"] = {k: v["hits"] for k, v in ops_.items() if v["hits"]}
            result["failures"] = {k: v["failures"] for k, v in ops_.items() if v["failures"]}
            result["fallbacks"] = {k: v["fallbacks"] for k, v in ops_.items() if v["fallbacks"]}
            result["declined"] = {k: v["declined"] for k, v in ops_.items() if v["declined"]}
            # share of the routed calls of the hooked ops that ran on the kernels
            calls = sum(v["hits"] + v["fallbacks"] for v in ops_.values())
            result["kernel_hit_fraction"] = round(sum(v["hits"] for v in ops_.values()) / calls, 5) if calls else None
        except Exception as exc:  # noqa: BLE001 - the counters are reported, not required
            result["usage_summary_error"] = str(exc)
    print("RESULT_JSON=" + json.dumps(result), flush=True)
    return 0


def launch(args, base: Path, model_dir: Path, gpus: str, tp: int, log: Path) -> subprocess.Popen:
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = gpus
    env["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0" if tp == 1 else "1"
    if tp > 1:
        # the per-rank counters are collected with collective_rpc on a plain function, which
        # vLLM serialises for its worker processes only with pickle allowed
        env["VLLM_ALLOW_INSECURE_SERIALIZATION"] = "1"
    paths = [str(ROOT)]
    if args.mode == "b200":
        paths += [str(write_plugin_dist(base)), str(PKG)]
        env["VLLM_PLUGINS"] = "vllm_nt"
        env["VLLM_NT_BACKEND_CONFIG"] = str(PKG / "vllm_nt" / "configs" / "all-b200.yaml")
        env["VLLM_NT_ENABLE_STATS"] = "1"
    else:
        env["VLLM_PLUGINS"] = ""
    env["PYTHONPATH"] = os.pathsep.join(paths + [env.get("PYTHONPATH", "")])
    cmd = [sys.executable, str(Path(__file__).resolve()), "--child", "--mode", args.mode, "--tp", str(tp),
           "--model-dir", str(model_dir), "--prompts", str(args.prompts), "--output-len", str(args.output_len),
           "--seed", str(args.seed), "--attention-backend", args.attention_backend, "--sampling", args.sampling]
    return subprocess.Popen(cmd, env=env, stdout=open(log, "w"), stderr=subprocess.STDOUT)


def parse_result(log: Path) -> dict | None:
    for line in log.read_text(errors="replace").splitlines()[::-1]:
        if line.startswith("RESULT_JSON="):
            return json.loads(line[len("RESULT_JSON="):])
    return None


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["b200", "native"], default="b200")
    ap.add_argument("--replicas", type=int, default=1)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--prompts", type=int, default=256)
    ap.add_argument("--output-len", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--log-dir", default="vllm_bench_logs", help="where each engine's log is written")
    ap.add_argument("--child", action="store_true")
    ap.add_argument("--model-dir")
    ap.add_argument("--attention-backend", default="FLASH_ATTN", choices=["FLASH_ATTN", "FLASHINFER"])
    ap.add_argument("--sampling", default="greedy", choices=["greedy", "topkp"],
                    help="greedy, or temperature 0.8 / top-k 50 / top-p 0.9 with a seed per request")
    args = ap.parse_args()
    if args.child:
        return child(args)

    base = Path(tempfile.mkdtemp(prefix="ntb200_e2e_"))
    model_dir = write_model_dir(base)
    logs = Path(args.log_dir)
    logs.mkdir(parents=True, exist_ok=True)
    procs = []
    if args.tp > 1:
        log = logs / f"vllm_{args.mode}_tp{args.tp}.log"
        procs.append((launch(args, base, model_dir, ",".join(str(i) for i in range(args.tp)), args.tp, log), log))
    else:
        for r in range(args.replicas):
            log = logs / f"vllm_{args.mode}_replica{r}.log"
            procs.append((launch(args, base, model_dir, str(r), 1, log), log))
    results = []
    for p, log in procs:
        p.wait(timeout=3000)
        res = parse_result(log)
        if p.returncode != 0 or res is None:
            print(json.dumps({"mode": args.mode, "error": f"engine failed (rc={p.returncode}), see {log}"}))
            return 1
        results.append(res)
    agg = {
        "metric": "vLLM offline output tok/s (Llama-3-8B-shaped, 256x512 in, 128 out, "
                  + ("greedy)" if args.sampling == "greedy" else "top-k 50 / top-p 0.9, seeded per request)"),
        "mode": args.mode,
        "replicas": len(results) if args.tp == 1 else 1,
        "tp": args.tp,
        "output_tok_s": sum(r["output_tok_s"] for r in results),
        "per_engine": results,
    }
    print(json.dumps(agg), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
