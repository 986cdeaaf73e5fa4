"""The allocation-free encoder entry point (czg_encode_intervals_static).

It serves callers that may not allocate device memory themselves (their device
memory belongs to another allocator), so its working storage is a fixed array
inside the library.  This test feeds it the coder intervals of real chunks,
with inputs and outputs in device memory the test owns, and checks that it
produces exactly the bytes of the regular compress entry point
(czg_compress_chunks), on two calls in a row: the second call reuses the array
with the first call's contents still in it.  The file sorts last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_static_encoder_matches_compress_entry(shipped_path, shipped_oracle, oracle_mod):
    import torch

    from compress_zip_b200 import czm, synth
    from compress_zip_b200 import engine as E

    mf = czm.ModelFile.load(shipped_path)
    tok = mf.tokenizer()
    eng = E.Engine(mf.raw, 0)
    try:
        for seed, C_len in ((3, 1024), (4, 200)):
            ids = np.array(tok.encode_with_special_tokens(synth.document(seed, 6000)), np.uint32)
            starts = np.array(list(range(0, len(ids), C_len)) + [len(ids)], np.uint64)
            lens = np.diff(starts).astype(np.uint32)
            want_packed, want_lens = eng.compress_packed(ids, starts)
            # and the CPU oracle's bytes for the same chunks, directly
            assert want_packed.tobytes() == b"".join(oracle_mod.compress_chunks(shipped_oracle, ids, starts))
            # coder intervals of every chunk from the GPU forward pass
            lohi = np.concatenate([eng.debug_trace(ids[int(a):int(b)])["lohi"]
                                   for a, b in zip(starts[:-1], starts[1:])]).astype(np.uint32)
            d_lohi = torch.from_numpy(lohi.view(np.int32)).cuda()
            d_len = torch.from_numpy(lens.view(np.int32)).cuda()
            cap = 4 * len(ids) + 8 * len(lens)
            stream = torch.cuda.current_stream().cuda_stream
            for call in range(2):
                d_out = torch.full((cap,), 0xAB, dtype=torch.uint8, device="cuda")
                d_out_lens = torch.zeros(len(lens), dtype=torch.int32, device="cuda")
                nbytes = C.c_uint64(0)
                st = E.lib().czg_encode_intervals_static(
                    d_lohi.data_ptr(), d_len.data_ptr(), len(lens), len(ids),
                    eng.info["target_total"], d_out.data_ptr(), cap, d_out_lens.data_ptr(),
                    C.byref(nbytes), C.c_void_p(stream))
                assert st == 0, f"call {call}: status {st}"
                assert nbytes.value == len(want_packed)
                got = d_out[: nbytes.value].cpu().numpy()
                assert np.array_equal(got, want_packed), f"call {call}: bytes differ"
                assert np.array_equal(d_out_lens.cpu().numpy().view(np.uint32), want_lens)
        # chunk lengths that do not add up to n_tokens: refused on the device before any
        # interval is read (CZG_E_ARG), nothing written
        for n_tok in (len(ids) - 1, len(ids) + 1):
            d_out.fill_(0xCD)
            nbytes = C.c_uint64(7)
            st = E.lib().czg_encode_intervals_static(
                d_lohi.data_ptr(), d_len.data_ptr(), len(lens), n_tok, eng.info["target_total"],
                d_out.data_ptr(), cap, d_out_lens.data_ptr(), C.byref(nbytes), C.c_void_p(stream))
            assert st == 1 and nbytes.value == 0
            assert bool((d_out == 0xCD).all())
        # beyond the stated limit: a clear status, no work
        nbytes = C.c_uint64(0)
        st = E.lib().czg_encode_intervals_static(
            d_lohi.data_ptr(), d_len.data_ptr(), 16385, 10, eng.info["target_total"],
            d_out.data_ptr(), cap, d_out_lens.data_ptr(), C.byref(nbytes), None)
        assert st == 9
    finally:
        eng.close()
