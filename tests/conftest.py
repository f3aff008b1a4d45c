import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _built(path, builder):
    if not os.path.exists(path):
        builder()
    return path


@pytest.fixture(scope="session")
def igc_lib():
    import igllm_b200
    from igllm_b200 import build
    _built(igllm_b200.LIB_PATH, build.build)
    return igllm_b200


@pytest.fixture(scope="session")
def igo_mod():
    import igo
    _built(igo.IGO_LIB, igo.build)
    return igo


TINY = dict(vocab=512, hidden=128, layers=7, heads=2, kv_heads=1, head_dim=64, inner=256, ple_dim=32,
            slide_span=8, share_count=2, global_every=3, window_limit=256, norm_offset=1.0,
            with_layer_scalar=1, seed=7)

# Wider than one 64-column chunk in every direction, 8 query heads against 1
# key/value head like the export, a window the block straddles, and ple_dim 32
# (a half chunk, so the padded-column path of the projections runs).
SMALL = dict(vocab=4096, hidden=256, layers=8, heads=8, kv_heads=1, head_dim=32, inner=512, ple_dim=32,
             slide_span=16, share_count=3, global_every=4, window_limit=512, norm_offset=1.0,
             with_layer_scalar=1, seed=11)

# The export's literal norm distribution, N(0, 0.02) used as is.
LITERAL = dict(TINY, norm_offset=0.0, with_layer_scalar=0, seed=3)

# A feed-forward wider than 2048 columns: above four lanes its down
# projection runs as side-by-side batches of four lanes in one launch.
WIDE = dict(TINY, inner=4096, seed=13)


# The export's head width (256) and 8:1 grouping at a size the reference
# primes in seconds, with every owner's key and value cache scales written
# (1/32 x 1, 1.125, 1.25, 1.375 by layer) for the 8-bit cache.  Layers 0-3
# are sliding owners with 64-row rings, 4 the global owner, 5 the last
# sliding owner (held full length for its sharers 6-8), 9 a global sharer.
CACHED = dict(vocab=8192, hidden=512, layers=10, heads=8, kv_heads=1, head_dim=256, inner=1024, ple_dim=64,
              slide_span=64, share_count=4, global_every=5, window_limit=1024, norm_offset=1.0,
              with_layer_scalar=1, seed=17, cache_scale_k=1.0 / 32, cache_scale_v=1.0 / 32)
# the shipped export's shape: global layers with a head of 512 and the doubled
# feed-forward on the sharing layers
EXPORT = dict(CACHED, global_head_dim=512, double_wide=1, seed=29)
# its stored forms: 2-bit late feed-forward codes, BF16 scales per 64
# columns, quantized embeddings, the embedding as the head
STORED = dict(EXPORT, late_mlp_bits=2, group=64, bf16_scales=1, embed_bits=2, ple_embed_bits=4, tied_head=1,
              seed=31)
# and the forms the tiles do not hold: 8-bit per-layer input planes, a dense
# per-layer model projection, activation grids on every projection
PLAIN = dict(STORED, ple_bits8=1, dense_ple_lift=1, grid_in=0.05, grid_out=0.02, seed=37)


def make_checkpoint(lib, folder, cfg):
    spec = lib.SynthSpec(**cfg)
    if not os.path.exists(os.path.join(folder, "model.safetensors")):
        lib.synth_write(spec, folder, 4)
    return spec


@pytest.fixture(scope="session")
def tiny_dir(tmp_path_factory, igc_lib):
    d = str(tmp_path_factory.mktemp("tiny"))
    make_checkpoint(igc_lib, d, TINY)
    return d


@pytest.fixture(scope="session")
def small_dir(tmp_path_factory, igc_lib):
    d = str(tmp_path_factory.mktemp("small"))
    make_checkpoint(igc_lib, d, SMALL)
    return d


@pytest.fixture(scope="session")
def literal_dir(tmp_path_factory, igc_lib):
    d = str(tmp_path_factory.mktemp("literal"))
    make_checkpoint(igc_lib, d, LITERAL)
    return d


@pytest.fixture(scope="session")
def wide_dir(tmp_path_factory, igc_lib):
    d = str(tmp_path_factory.mktemp("wide"))
    make_checkpoint(igc_lib, d, WIDE)
    return d


@pytest.fixture(scope="session")
def cached_dir(tmp_path_factory, igc_lib):
    d = str(tmp_path_factory.mktemp("cached"))
    make_checkpoint(igc_lib, d, CACHED)
    return d
