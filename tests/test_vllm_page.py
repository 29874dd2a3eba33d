"""Layout of the vLLM memory page (vllm_yanchor.py:19-62) as seen through
``state_from_vllm_page``: every field is a view of the page at the plugin's
offsets, with the plugin's bit-casts (int32 positions, int64 count / total
inside the float32 meta page).  CPU only: no kernel runs."""
import torch

from yanchor_b200 import independent_memory as im


def test_views_alias_the_page_at_the_plugins_offsets():
    G, CAP, CH, D, P = 4, 64, 64, 256, 3
    vs, ms = im.vllm_page_shapes(G, CAP, CH, D)
    assert vs == (2 * G * (CAP + CH) * D,) and ms == (G * (2 * CAP + CH) + 4,)
    values = torch.zeros((P,) + vs, dtype=torch.bfloat16)
    meta = torch.zeros((P,) + ms)
    st = im.state_from_vllm_page(values, meta, G, CAP, CH, D)
    im._check_state(st)
    st.keys[1, 2, 3, 4] = 1.5
    assert values[1, (2 * CAP + 3) * D + 4] == 1.5
    st.pending_values[2, 0, 1, 0] = -2.0
    assert values[2, (2 * G * CAP + G * CH + 1) * D] == -2.0
    st.positions[0, 1, 2] = 77
    assert meta[0, G * CAP + CAP + 2].view(torch.int32).item() == 77
    st.count[2] = 5
    st.total[2] = 2**40
    assert meta[2, -4:-2].view(torch.int64).item() == 5 and meta[2, -2:].view(torch.int64).item() == 2**40
    im.reset_vllm_page_(st, torch.tensor([2]))
    assert st.count[2] == 0 and st.total[2] == 0 and bool((st.positions[2] == -1).all())
    assert bool(torch.isinf(st.scores[2]).all()) and st.keys[1, 2, 3, 4] == 1.5    # other pages untouched
