"""Attaching the prefill hook to the installed vLLM (0.22) on the CPU: the anchor-based source patch
on a copy of vLLM's flash_attn.py, and the runtime wrapper's routing (which calls reach
try_sparse_forward, and that a False return falls through to vLLM's own forward)."""
import importlib.util
import shutil
import types
from pathlib import Path

import pytest
import torch

VLLM = importlib.util.find_spec('vllm')
pytestmark = pytest.mark.skipif(VLLM is None, reason='vllm is not installed')


def _vllm_dir() -> Path:
    return Path(list(VLLM.submodule_search_locations)[0])


def test_patch_source_on_a_copy(tmp_path):
    from sm120_attn import vllm_hook as vh
    src = _vllm_dir() / 'v1' / 'attention' / 'backends' / 'flash_attn.py'
    dst = tmp_path / 'v1' / 'attention' / 'backends' / 'flash_attn.py'
    dst.parent.mkdir(parents=True)
    shutil.copy(src, dst)
    before = dst.read_text()
    assert vh.patch_source(tmp_path, check=True) == 'would patch'
    assert dst.read_text() == before                                  # --check changes nothing
    assert vh.main(['--target', str(tmp_path)]) == 0
    after = dst.read_text()
    assert 'try_sparse_forward(' in after and after.count('try_sparse_forward(') == 1
    compile(after, str(dst), 'exec')                                  # still valid Python
    assert vh.patch_source(tmp_path) == 'already patched'
    dst.write_text(before.replace(vh.ANCHOR, ''))
    assert vh.patch_source(tmp_path).startswith('ANCHOR NOT FOUND')
    with pytest.raises(FileNotFoundError):
        vh.patch_source(tmp_path / 'nowhere')


def _impl_class(calls):
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        calls.append('vllm')
        return output
    return type('StubImpl', (FlashAttentionImpl,), {'forward': forward})


def test_runtime_install_routes_calls(monkeypatch):
    from vllm.v1.attention.backend import AttentionType
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn import vllm_hook as vh
    calls, seen = [], []
    answer = {'value': True}

    def fake_try(impl, query, key, key_cache, value_cache, output, meta):
        seen.append((query.shape, key.shape, key_cache.data_ptr(), value_cache.data_ptr(), output.shape))
        calls.append('sparse')
        return answer['value']
    monkeypatch.setattr(ksp, 'try_sparse_forward', fake_try)
    cls = _impl_class(calls)
    assert vh.install(cls) is True and vh.install(cls) is False       # idempotent
    impl = object.__new__(cls)
    impl.attn_type, impl.kv_cache_dtype, impl.dcp_world_size = AttentionType.DECODER, 'auto', 1
    kv_cache = torch.zeros(2, 3, 16, 2, 8)
    q, k, v, out = torch.zeros(7, 4, 8), torch.zeros(7, 2, 8), torch.zeros(7, 2, 8), torch.zeros(7, 4, 8)
    meta = types.SimpleNamespace(num_actual_tokens=5, use_cascade=False)

    assert impl.forward(None, q, k, v, kv_cache, meta, out) is out  # handled by the sparse path
    assert calls == ['sparse']
    assert seen[0] == ((5, 4, 8), (5, 2, 8), kv_cache[0].data_ptr(), kv_cache[1].data_ptr(), (5, 4, 8))
    answer['value'] = False                                          # not eligible: vLLM's path runs
    impl.forward(None, q, k, v, kv_cache, meta, out)
    assert calls == ['sparse', 'sparse', 'vllm']
    calls.clear()
    impl.forward(None, q, k, v, kv_cache, None, out)                 # profiling run
    impl.kv_cache_dtype = 'fp8'                                      # quantised cache
    impl.forward(None, q, k, v, kv_cache, meta, out)
    impl.kv_cache_dtype = 'auto'
    impl.forward(None, q, k, v, kv_cache, types.SimpleNamespace(num_actual_tokens=5, use_cascade=True), out)
    impl.attn_type = AttentionType.ENCODER_ONLY
    impl.forward(None, q, k, v, kv_cache, meta, out)
    assert calls == ['vllm'] * 4                                     # none of these reach the hook
    assert vh.uninstall(cls) is True and vh.uninstall(cls) is False
    calls.clear()
    impl.attn_type = AttentionType.DECODER
    impl.forward(None, q, k, v, kv_cache, meta, out)
    assert calls == ['vllm']                                         # the original forward is back
