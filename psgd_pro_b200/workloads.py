"""Parameter sets of the benchmark configurations (shapes in nn.Linear (out, in) layout, parameter dtype, gradient
scale). The parameters are synthetic: random-init values of these shapes stand in for the named models, and
gradients are N(0, std^2) draws of these shapes (no datasets or checkpoints are read)."""


def vit_tiny():
    """ViT-Tiny of the reference demo (vit_pro.py:157-225, dim 192, depth 12, 3 heads of 64, MLP 768, patch 4,
    3 x 32 x 32 input, 10 classes): 144 tensors, 5.36 M parameters."""
    d, mlp, inner, pd = 192, 768, 192, 48
    s = [(pd,), (pd,), (d, pd), (d,), (d,), (d,), (1, 65, d), (1, 1, d)]
    for _ in range(12):
        s += [(d,), (d,), (3 * inner, d), (d, inner), (d,)]
        s += [(d,), (d,), (mlp, d), (mlp,), (d, mlp), (d,)]
    s += [(d,), (d,), (10, d), (10,)]
    return s


def gpt2_medium():
    """GPT-2 medium (24 layers, d 1024, MLP 4096, vocab 50257, context 1024, tied head): 292 tensors, 354.8 M."""
    d, f = 1024, 4096
    s = [(50257, d), (1024, d)]
    for _ in range(24):
        s += [(d,), (d,), (3 * d, d), (3 * d,), (d, d), (d,), (d,), (d,), (f, d), (f,), (d, f), (d,)]
    s += [(d,), (d,)]
    return s


def llama_1b():
    """Llama-style 1.1 B (d 2048, 22 layers, FFN 5632, 32 heads with 4 KV heads of 64, vocab 32000, untied head):
    201 tensors, 1.100 B parameters."""
    d, f, kv = 2048, 5632, 256
    s = [(32000, d)]
    for _ in range(22):
        s += [(d, d), (kv, d), (kv, d), (d, d), (f, d), (f, d), (d, f), (d,), (d,)]
    s += [(d,), (32000, d)]
    return s


def llama_layer():
    """One decoder layer of the Llama-style set (the same factor sizes 256, 2048 and 5632): a small case of the
    1.1 B workload for profiling, 9 tensors, 44 M parameters."""
    d, f, kv = 2048, 5632, 256
    return [(d, d), (kv, d), (kv, d), (d, d), (f, d), (f, d), (d, f), (d,), (d,)]


def config1():
    """One fp32 256 x 512 weight (the reference CPU case)."""
    return [(256, 512)]


WORKLOADS = {
    # name: (shapes, parameter dtype, gradient dtype, gradient std, description)
    "llama-1.1b": (llama_1b, "bf16", "bf16", 1e-3, "Llama-style 1.1B parameter set, bf16 params/grads, fp32 Q"),
    "llama-layer": (llama_layer, "bf16", "bf16", 1e-3, "one decoder layer of the Llama-style set (profiling case)"),
    "gpt2-medium": (gpt2_medium, "bf16", "bf16", 1e-3, "GPT-2-medium parameter set, bf16 params/grads, fp32 Q"),
    "vit-tiny": (vit_tiny, "fp32", "bf16", 1e-3, "ViT-Tiny parameter set, fp32 params, bf16 grads"),
    "config1": (config1, "fp32", "fp32", 1e-2, "one fp32 256x512 weight"),
}
