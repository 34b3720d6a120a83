"""The vLLM prefill hook for the installed vLLM (0.22): runtime install or anchor-based source patch.

The reference inserts `try_sparse_forward` into vLLM's FlashAttention backend by matching a source
anchor of its vLLM version (tools/patch_vllm.py:18-30), after which `FlashAttentionImpl.forward`
hands long causal prefill chunks to the sparse path and runs flash_attn_varlen_func for the rest.
vLLM 0.22 no longer contains that anchor: its forward no longer branches on `attn_metadata.causal`
there, and the KV cache is written before forward by `do_kv_cache_update`.  Two equivalent ways to
attach the same hook to 0.22:

* `install()` wraps `FlashAttentionImpl.forward` at run time (idempotent; `uninstall()` restores
  it).  Call it once in every worker process before the model runs, e.g. from a vLLM general
  plugin entry point.
* `patch_source(target)` / `python -m sm120_attn.vllm_hook --target <vllm package dir> [--check]`
  inserts the hook into v1/attention/backends/flash_attn.py by anchor matching, like the
  reference's patcher (idempotent; reports ANCHOR NOT FOUND for other vLLM versions).

Either way the hook runs only where the reference's does: decoder self-attention, no cascade
attention, no decode-context parallelism and an unquantised KV cache; `try_sparse_forward` then
applies the SM120_SPARSE_* gates (causal, no sliding window, min_q / min_kv, not during CUDA graph
capture) and returns False, leaving vLLM's own path to run, for everything else.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

_ORIGINAL = '_sm120_sparse_original_forward'


def _flash_attn_impl():
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl
    return FlashAttentionImpl


def _eligible_call(impl, attn_metadata, output_scale, output_block_scale) -> bool:
    """Host-side conditions under which the reference's hook point is reached in 0.22's forward."""
    if attn_metadata is None or output_scale is not None or output_block_scale is not None:
        return False
    from vllm.v1.attention.backend import AttentionType
    if getattr(impl, 'attn_type', AttentionType.DECODER) != AttentionType.DECODER:
        return False
    if getattr(attn_metadata, 'use_cascade', False) or getattr(impl, 'dcp_world_size', 1) > 1:
        return False
    from vllm.utils.torch_utils import is_quantized_kv_cache
    return not is_quantized_kv_cache(getattr(impl, 'kv_cache_dtype', 'auto'))


def install(impl_cls=None) -> bool:
    """Wrap `impl_cls.forward` (default: vLLM's FlashAttentionImpl) with the sparse prefill hook.
    Returns False when it is already installed."""
    cls = impl_cls if impl_cls is not None else _flash_attn_impl()
    if _ORIGINAL in cls.__dict__:
        return False
    original = cls.forward

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if _eligible_call(self, attn_metadata, output_scale, output_block_scale):
            from .sparse_prefill import try_sparse_forward
            n = attn_metadata.num_actual_tokens
            key_cache, value_cache = kv_cache.unbind(0)
            if try_sparse_forward(self, query[:n], key[:n], key_cache, value_cache, output[:n], attn_metadata):
                return output
        return original(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                        output_block_scale)

    forward.__doc__ = original.__doc__
    forward.__wrapped__ = original
    setattr(cls, _ORIGINAL, original)
    cls.forward = forward
    return True


def uninstall(impl_cls=None) -> bool:
    cls = impl_cls if impl_cls is not None else _flash_attn_impl()
    original = cls.__dict__.get(_ORIGINAL)
    if original is None:
        return False
    cls.forward = original
    delattr(cls, _ORIGINAL)
    return True


# vLLM 0.22 v1/attention/backends/flash_attn.py: the non-DCP branch of the non-cascade path, right
# before flash_attn_varlen_func (the KV cache already holds this step's keys and values).
ANCHOR = """            else:
                sliding_window_size = (
"""
HOOK = """            else:
                # dynamic block-sparse attention for long prefill chunks (sm120_attn)
                from sm120_attn.sparse_prefill import try_sparse_forward
                if not is_quantized_kv_cache(self.kv_cache_dtype) and try_sparse_forward(
                        self, query[:num_actual_tokens], key[:num_actual_tokens], key_cache, value_cache,
                        output[:num_actual_tokens], attn_metadata):
                    return output
                sliding_window_size = (
"""


def patch_source(target: Path, check: bool = False) -> str:
    """Insert the hook into <target>/v1/attention/backends/flash_attn.py (target: the vllm package
    directory).  Returns 'patched', 'would patch', 'already patched' or 'ANCHOR NOT FOUND ...'."""
    fa = Path(target) / 'v1' / 'attention' / 'backends' / 'flash_attn.py'
    if not fa.exists():
        raise FileNotFoundError(f'{fa} not found: target must be the vllm package directory')
    text = fa.read_text()
    if HOOK in text:
        return 'already patched'
    if text.count(ANCHOR) != 1:
        return 'ANCHOR NOT FOUND (vLLM version mismatch?)'
    if not check:
        fa.write_text(text.replace(ANCHOR, HOOK, 1))
    return 'would patch' if check else 'patched'


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description='attach the sparse prefill hook to an installed vLLM 0.22')
    ap.add_argument('--target', type=Path, required=True, help='directory of the vllm package')
    ap.add_argument('--check', action='store_true', help='report without changing anything')
    args = ap.parse_args(argv)
    result = patch_source(args.target, args.check)
    print('flash_attn.py:', result)
    return 0 if not result.startswith('ANCHOR') else 1


if __name__ == '__main__':
    sys.exit(main())
