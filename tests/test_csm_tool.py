"""`.csm` v1 writer / reader round trip and checkpoint layout (no GPU)."""
import numpy as np


def test_roundtrip_and_names(make_csm):
    import csm_tool

    path = make_csm("tiny2", seed=3)
    cfg, t = csm_tool.read_csm(path)
    assert cfg["dim"] == 128 and cfg["num_stems"] == 2 and cfg["time_transformer_depth"] == 2
    assert t["__precomputed__.freq_indices"].dtype == np.int64
    assert t["layers.1.0.layers.1.0.to_qkv.weight"].shape == (3 * 2 * 64, 128)
    assert t["mask_estimators.1.to_freqs.59.0.4.weight"].shape[1] == 512
    # the same seed gives the same checkpoint
    again = csm_tool.random_weights(csm_tool.base_config(**csm_tool.PRESETS["tiny2"]), 3)
    for k, v in again.items():
        assert np.array_equal(v, t[k]), k


def test_oracle_reads_writer_output(make_csm):
    import oracle

    m = oracle.Model(make_csm("tiny", seed=4))
    assert m.info("dim") == 64 and m.info("band_freqs") == 3958 and m.info("channels") == 2
