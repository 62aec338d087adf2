"""SGLang general-plugin entry point (stepquant/sglang/plugin.py).

``register()`` installs AROUND hooks through SGLang's HookRegistry for the
packed state pool, the GDN/KDA kernels, the model runner checks, pool sizing,
and (with STEPQUANT_ASYNC_WRITEBACK=1) the graph capture and attention release
windows.  It is a no-op unless STEPQUANT_PLAN or STEPQUANT_STATE_FORMAT is set.
"""
import os

PINNED_SGLANG = "0.5.12"


def hook_targets(environ=None):
    """(sglang target path, runtime function name) pairs that register() installs."""
    env = os.environ if environ is None else environ
    targets = []
    pool = "mem_cache.memory_pool.MambaPool."
    for method in ("__init__", "alloc", "copy_from", "get_cpu_copy", "load_cpu_copy", "get_contiguous_buf_infos"):
        targets.append((pool + method, "pool_" + method.strip("_")))
    for cls, architecture in (("gdn_triton.TritonGDNKernel", "gdn"), ("kda_triton.TritonKDAKernel", "kda")):
        prefix = "layers.attention.linear.kernels." + cls + "."
        targets.append((prefix + "decode", "kernel_decode"))
        targets.append((prefix + "extend", "kernel_extend"))
        if architecture == "gdn":
            targets.append((prefix + "packed_decode", "kernel_packed_decode"))
    targets.append(("model_executor.model_runner.ModelRunner.__init__", "validate_runner"))
    targets.append(("model_executor.model_runner_kv_cache_mixin.ModelRunnerKVCacheMixin.handle_max_mamba_cache",
                    "size_pool"))
    if env.get("STEPQUANT_ASYNC_WRITEBACK") == "1":
        targets.append(("model_executor.cuda_graph_runner.CudaGraphRunner.capture_one_batch_size", "capture_graph"))
        if env.get("STEPQUANT_ARCHITECTURE") == "kda":
            targets.append(("models.kimi_linear.KimiDecoderLayer.forward", "attention_forward"))
        else:
            for cls in ("Qwen3_5LinearDecoderLayer", "Qwen3_5AttentionDecoderLayer"):
                targets.append(("models.qwen3_5." + cls + ".forward", "attention_forward"))
    return targets


def verify_hooks():
    """Refuse to run if any installed STEPQuant hook was not patched (no silent FP32 fallback)."""
    from sglang.srt.plugins.hook_registry import HookRegistry
    required = [target for target, hooks in HookRegistry._hooks.items()
                if any(getattr(fn, "__module__", "") == "stepquant_b200.sglang.runtime" for _, fn, _ in hooks)]
    missing = set(required) - HookRegistry._patched
    if not required or missing:
        raise RuntimeError(f"STEPQuant plugin hooks incomplete: {sorted(missing)}; refusing FP32 fallback")


def register():
    if not (os.environ.get("STEPQUANT_PLAN") or os.environ.get("STEPQUANT_STATE_FORMAT")):
        return
    from importlib.metadata import version
    if version("sglang") != PINNED_SGLANG:
        raise RuntimeError(f"STEPQuant integration is pinned to sglang=={PINNED_SGLANG}")
    from sglang.srt.plugins.hook_registry import HookRegistry, HookType
    from . import runtime
    for target, name in hook_targets():
        HookRegistry.register("sglang.srt." + target, getattr(runtime, name), HookType.AROUND)
