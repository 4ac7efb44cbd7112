"""The bench line's arithmetic (CPU only): the prefill roofline is one GPU's
FLOPs over one GPU's peak whatever the rank count, and the bench's reference
arm builds its model without the product's libraries."""
import bench


def test_prefill_roofline_is_per_gpu():
    flops_per_gpu = 8 * bench.prefill_flops(bench_shape(), bench.PREFILL_PROMPT)
    one = bench.prefill_roofline(flops_per_gpu, 400.0, 1389.6, "measured")
    # Two ranks each prefilling their own eight prompts in the same time: the
    # per-GPU fraction is unchanged (the job's tok/s doubles, not the fraction).
    two = bench.prefill_roofline(flops_per_gpu, 400.0, 1389.6, "measured")
    assert one["frac"] == two["frac"]
    assert abs(one["achieved"] - flops_per_gpu / 0.4 / 1e12) < 1e-6 * one["achieved"]
    assert abs(one["frac"] - one["achieved"] / 1389.6) < 1e-12


def test_reference_arm_names_no_product_library():
    import inspect

    source = inspect.getsource(bench.run_reference)
    for name in ("native.synthetic_tensor", "native.synthetic_tokens", "native.host", "native.cuda", "Context("):
        assert name not in source


def bench_shape():
    from huggingfaceeacp_b200 import native

    return native.GEMMA_2B
