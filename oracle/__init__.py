"""CPU oracle for the Laguna MoE block and the 8-bit KV decode attention.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker (or the timed CPU baseline). The product path
(``lagunalab_b200``) never imports it and has no CPU fallback.

Every function restates the reference algorithm and cites the reference file and
line it follows (paths relative to the lagunaLab project root):

* ``mlx_quant``  MLX affine quantization layout: uint32 words, low bits first,
  bf16 scale/bias per group (laguna_mlx/q8_attn.py:8-10, :50, :55;
  scripts/pack_experts.py:19-30).
* ``moe_ref``    router, SwitchGLU, shared MLP and the block combine
  (laguna_mlx/laguna.py:114-150), with the bf16 materialisation points of the
  MLX graph.
* ``attn_ref``   the fused q8 decode attention (laguna_mlx/q8_attn.py:17-130)
  and the quantized KV cache append rules (laguna_mlx/cache.py:66-145).

Parity pins: the unquantized router / experts / block are pinned against the
reference's vendored PyTorch model (tests/reference/modeling_laguna.py:146-266)
through the golden fixtures in ``tests/golden`` (made by
``tests/golden/make_golden.py``). The 4-bit ``gather_qmm`` rounding inside
mlx 0.32.0 cannot be run here (MLX is not installable), so the quantized path
is pinned only through the dequantization formula and the packed layouts.
"""
