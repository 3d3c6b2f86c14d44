"""PackedWeightLoader on the GPU: quantize + pack with the reference's padding,
dequantize bit-exactly against the oracle, save and reload through the safetensors
file, and run the GEMM on a reloaded stream."""

import numpy as np
import pytest

from oracle import int4 as O

pytestmark = pytest.mark.gpu


def test_loader_round_trip_and_gemm(cuda, tmp_path):
    import torch
    from moat_b200.gemm import batched_gemm
    from moat_b200.packed import PackedWeightLoader
    K, M = 512, 768
    w = O.make_weights(K, M, 21).astype(np.float16)
    odd = O.make_weights(1, 300, 22).astype(np.float16)  # 300 elements: padded to 512
    ld = PackedWeightLoader(device=str(cuda))
    lay = ld.load_and_repack_layer("proj", w)
    ld.load_and_repack_layer("odd", odd.reshape(300))
    assert lay["memory_bytes"] == K * M // 256 * 144 and ld.total_loaded_bytes == lay["memory_bytes"] + 2 * 144
    # bit-exact against the oracle's engine quantizer + packer + dequant
    st = O.quantize_pack_matrix(w.astype(np.float32))
    np.testing.assert_array_equal(lay["superblocks"].cpu().numpy(), st)
    deq = ld.dequantize_layer("proj")
    np.testing.assert_array_equal(deq.cpu().numpy().view(np.uint16),
                                  O.unpack_superblock_weights(st).reshape(K, M).view(np.uint16))
    od = ld.dequantize_layer("odd")
    assert tuple(od.shape) == (300,)
    pad = np.zeros(512, np.float32)
    pad[:300] = odd.reshape(300).astype(np.float32)
    ref_odd = O.unpack_superblock_weights(O.quantize_pack_matrix(pad.reshape(2, 256)))[:300]
    np.testing.assert_array_equal(od.cpu().numpy().view(np.uint16), ref_odd.view(np.uint16))
    # save, reload into a fresh loader, same bytes, GEMM equal bit for bit
    p = str(tmp_path / "model.safetensors")
    ld.save(p)
    ld2 = PackedWeightLoader(device=str(cuda))
    ld2.load(p)
    assert torch.equal(ld2.layers["proj"]["superblocks"], lay["superblocks"])
    assert ld2.layers["odd"]["n_elements"] == 300 and ld2.layers["odd"]["original_shape"] == (300,)
    x = torch.from_numpy(O.make_activations(4, K, 5)).cuda()
    y1 = batched_gemm(x, lay["superblocks"], K, M)
    y2 = batched_gemm(x, ld2.layers["proj"]["superblocks"], K, M)
    assert torch.equal(y1, y2)
    with pytest.raises(MemoryError):
        PackedWeightLoader(memory_budget_bytes=1000, device=str(cuda)).load_and_repack_layer("big", w)
