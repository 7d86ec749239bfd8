"""One vLLM engine run for test_e2e_vllm_gpu.py (prints one JSON line).

``python tests/e2e_vllm_worker.py <stock|stock_flash_attn|custom> <prompt_len> <new_tokens> <split> [layers]``

Model: the Qwen2.5-7B attention/MLP geometry (28 / 4 heads, head_dim 128,
hidden 3584, SwiGLU 18944, RoPE theta 1e6) with 2 layers (or ``layers``), from the config in
``tests/e2e/qwen2_7b_geometry`` - no checkpoint: vLLM's dummy loader, then
every weight re-drawn from a seeded N(0, 0.02) (norm weights 1), identically
in every run, so the logits are not near-uniform.  ``stock`` runs vLLM's own
attention backend; ``custom`` registers this package and runs the CUSTOM
backend with ``HCP_RING_SPLIT_TOKENS=<split>``.  Greedy decoding, top-2
logprobs per step.
"""

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
CFG = os.path.join(HERE, "e2e", "qwen2_7b_geometry")


def reinit(model):
    import torch
    g = torch.Generator(device="cuda").manual_seed(1234)
    n = 0
    with torch.no_grad():
        for name, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
            if p.dim() == 1 and "norm" in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02, generator=g)
            n += p.numel()
    return n


def main():
    mode, prompt_len, new_tokens, split = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4])
    layers = int(sys.argv[5]) if len(sys.argv) > 5 else None
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    if mode == "custom":
        os.environ["HCP_RING_SPLIT_TOKENS"] = str(split)
        from hcp_vllm_plugin_b200 import register
        register()
    import numpy as np
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    kwargs = dict(model=CFG, dtype="bfloat16", load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
                  gpu_memory_utilization=0.5, max_model_len=max(8192, prompt_len + new_tokens + 16),
                  disable_hybrid_kv_cache_manager=True, seed=0, block_size=16)
    if layers is not None:
        kwargs["hf_overrides"] = {"num_hidden_layers": layers, "max_window_layers": layers}
    if mode == "custom":
        kwargs["attention_backend"] = "CUSTOM"
    elif mode == "stock_flash_attn":   # a second stock backend, as a control
        kwargs["attention_backend"] = "FLASH_ATTN"
    llm = LLM(**kwargs)
    params = llm.apply_model(reinit)[0]
    ids = np.random.default_rng(7).integers(0, 151000, size=prompt_len).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=new_tokens, logprobs=2, ignore_eos=True)
    import time
    t0 = time.perf_counter()
    res = llm.generate([TokensPrompt(prompt_token_ids=ids)], sp)[0].outputs[0]
    gen_s = time.perf_counter() - t0
    margins = []
    for step in res.logprobs:
        top = sorted((lp.logprob for lp in step.values()), reverse=True)
        margins.append(float(top[0] - top[1]) if len(top) > 1 else float("inf"))
    out = {"mode": mode, "split": split, "params": int(params), "tokens": list(res.token_ids), "margins": margins,
           "generate_s": gen_s}
    if mode == "custom":
        from hcp_vllm_plugin_b200 import ring_backend as rb
        out["impl_stats"] = dict(rb.IMPL_STATS)
    print("E2E_RESULT " + json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
