"""vLLM 0.22 serving a tiny random-weight Llama (head_dim 128) in-process, with the sparse prefill hook
attached by `sm120_attn.vllm_hook.install()`.  Run by tests/test_zy_vllm_e2e.py in a subprocess;
prints one JSON line.

A 3000-token prompt is prefilled in 2048-token chunks by vLLM's scheduler with its FlashAttention
backend.  Three runs of greedy decoding (4 tokens, top-5 logprobs of the first):
  hooked_bf16  hook installed, BF16 kernel, tau 1 (every block kept: dense attention)
  vllm         hook uninstalled (vLLM's own flash_attn_varlen_func)
  hooked_fp8   hook installed, FP8 kernel, tau 0.95 (sparse selection)
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(ROOT / 'qwen38-sparse-attn_b200')]
os.environ.setdefault('VLLM_ENABLE_V1_MULTIPROCESSING', '0')
for k, v in {'SM120_SPARSE_ATTN': '1', 'SM120_SPARSE_MIN_KV': '1024', 'SM120_SPARSE_MIN_Q': '512'}.items():
    os.environ[k] = v


def tiny_model(path: Path):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=1024, hidden_size=1024, intermediate_size=2048, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=8192,
                      rope_theta=1e6, torch_dtype='bfloat16', tie_word_embeddings=False, bos_token_id=1, eos_token_id=2)
    torch.manual_seed(0)
    LlamaForCausalLM(cfg).to(torch.bfloat16).save_pretrained(path, safe_serialization=True)


def main():
    import torch
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn import vllm_hook
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt
    with tempfile.TemporaryDirectory() as tmp:
        tiny_model(Path(tmp))
        llm = LLM(model=tmp, skip_tokenizer_init=True, enforce_eager=True, max_model_len=4096, dtype='bfloat16',
                  gpu_memory_utilization=0.3, max_num_batched_tokens=2048, seed=0, attention_backend='FLASH_ATTN',
                  enable_prefix_caching=False)          # every run prefills the whole prompt
        ids = torch.randint(3, 1000, (3000,), generator=torch.Generator().manual_seed(0)).tolist()
        sp = SamplingParams(max_tokens=4, temperature=0.0, logprobs=5, detokenize=False)

        def run(kernel=None, tau=None):
            if kernel is not None:
                os.environ['SM120_SPARSE_KERNEL'], os.environ['SM120_SPARSE_TAU'] = kernel, tau
                ksp._CONFIG = None
                ksp._STATE.clear()
            out = llm.generate([TokensPrompt(prompt_token_ids=ids)], sp, use_tqdm=False)[0].outputs[0]
            calls = sum(s.stats['calls'] for s in ksp._STATE.values())
            return {'tokens': list(out.token_ids), 'logprobs': {int(t): float(v.logprob) for t, v in out.logprobs[0].items()},
                    'sparse_calls': calls}

        res = {'installed': vllm_hook.install()}
        res['hooked_bf16'] = run('sm120', '1.0')
        vllm_hook.uninstall()
        ksp._STATE.clear()
        res['vllm'] = run()
        vllm_hook.install()
        res['hooked_fp8'] = run('sm120fp8', '0.95')
        vllm_hook.uninstall()
    print('RESULT ' + json.dumps(res), flush=True)


if __name__ == '__main__':
    main()
