"""tc_conv_w8a8_noalloc, the convolution entry point for callers that cannot let the library
allocate device memory during a call, against the CPU oracle's conv descriptor and against the
regular conv path (the same descriptor through the drop-in Machine): identical output bytes on
three calls in a row - 63 output rows (tensor-core GEMM), then 4 rows (the M <= 8 GEMV) and 12 rows
(the generic GEMV) after it, so a smaller gather reuses the fixed buffer that a larger one filled
and stale bytes would show. This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

from oracle import contract as C

pytestmark = pytest.mark.gpu


# (H, W, KH, KW, stride, pad, Cin, N): OH*OW = 63, 4 and 12 output rows
SHAPES = [(9, 7, 3, 3, 1, 1, 32, 48), (4, 4, 3, 3, 2, 1, 32, 32), (6, 8, 3, 3, 2, 1, 16, 64)]


def _case(seed):
    rng = np.random.default_rng(seed)
    H, W, KH, KW, S, P, cin, N = SHAPES[seed]
    OH, OW = (H + 2 * P - KH) // S + 1, (W + 2 * P - KW) // S + 1
    K = KH * KW * cin
    img = rng.integers(-128, 128, (H * W, cin), dtype=np.int8)
    w = rng.integers(-128, 128, (N, K), dtype=np.int8)
    sc = rng.uniform(1e-4, 1e-2, N).astype("<f4")
    bias = rng.normal(0, 1, N).astype("<f4")
    return dict(H=H, W=W, KH=KH, KW=KW, S=S, P=P, cin=cin, N=N, OH=OH, OW=OW, K=K, img=img, w=w, sc=sc, bias=bias,
                act=C.ACT_GELU, out=C.OUT_FP32)


def _conv_program(c):
    """The same convolution as one conv descriptor in a DDR image."""
    ddr = bytearray(1 << 20)
    a_off, w_off, s_off, b_off, y_off, qa = 0x1000, 0x10000, 0x40000, 0x41000, 0x50000, 0xF0000
    ddr[a_off:a_off + c["img"].size] = c["img"].tobytes()
    ddr[w_off:w_off + c["w"].size] = c["w"].tobytes()
    ddr[s_off:s_off + 4 * c["N"]] = c["sc"].tobytes()
    ddr[b_off:b_off + 4 * c["N"]] = c["bias"].tobytes()
    ddr[qa:qa + 64] = C.encode(dict(
        MAGIC=C.MAGIC, VERSION=C.VERSION, VALID=1, OPCODE=C.OP_CONV_ACT, CTRL=C.ctrl(C.QM_CHANNEL, fusion=1),
        EPI=C.epi(c["act"], c["out"], 1), A_OFF=a_off, W_OFF=w_off, SCALE_OFF=s_off, BIAS_OFF=b_off, Y_OFF=y_off,
        M=c["OH"] * c["OW"], N=c["N"], K=c["K"], GROUP_SIZE=c["W"],
        HDR_RSV=c["H"] << 12 | c["KH"] << 8 | c["KW"] << 4 | (c["S"] - 1) << 2 | c["P"]))
    return ddr, qa, slice(y_off, y_off + 4 * c["N"] * c["OH"] * c["OW"])


def _oracle_conv(c) -> bytes:
    from oracle.machine import OracleMachine
    ddr, qa, ys = _conv_program(c)
    m = OracleMachine(ddr)
    assert m.run_queue(qa, 1).done
    return bytes(m.ddr[ys])


def _machine_conv(c) -> bytes:
    from opentars_b200.machine import Machine
    ddr, qa, ys = _conv_program(c)
    m = Machine(ddr)
    assert m.run_queue(qa, 1).done
    return bytes(m.ddr[ys])


def test_noalloc_conv_matches_the_oracle_on_calls_in_a_row():
    import torch
    from opentars_b200._lib import lib
    L = lib()
    dev = torch.device("cuda", 0)
    for seed in range(len(SHAPES)):          # calls in a row: a large gather, then smaller ones
        c = _case(seed)
        want = _oracle_conv(c)
        assert _machine_conv(c) == want, seed
        img = torch.from_numpy(c["img"].view(np.uint8).copy()).to(dev)
        w = torch.from_numpy(c["w"].view(np.uint8).copy()).to(dev)
        sc = torch.from_numpy(c["sc"].copy()).to(dev)
        bias = torch.from_numpy(c["bias"].copy()).to(dev)
        y = torch.full((c["OH"] * c["OW"] * c["N"] * 4,), 0xAB, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        rc = L.tc_conv_w8a8_noalloc(img.data_ptr(), c["cin"], c["H"], c["W"], c["cin"], c["KH"], c["KW"], c["S"],
                                    c["P"], w.data_ptr(), sc.data_ptr(), 1, bias.data_ptr(), y.data_ptr(),
                                    4 * c["N"], c["N"], c["act"], c["out"], ctypes.c_float(0.0),
                                    ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0
        torch.cuda.synchronize(dev)
        assert y.cpu().numpy().tobytes() == want, seed


def test_noalloc_conv_rejects_oversized_and_bad_arguments():
    from opentars_b200._lib import TC_ERR_ARG, TC_ERR_TOO_LARGE, lib
    L = lib()
    fake = ctypes.c_void_p(16)                # never dereferenced: the checks come first
    # 1024 x 1024 pixels of 32 channels with a 3 x 3 window: 1M rows x 288 bytes > 16 MiB
    assert L.tc_conv_w8a8_noalloc(fake, 32, 1024, 1024, 32, 3, 3, 1, 1, fake, fake, 1, None, fake, 64, 16, 0, 0,
                                  ctypes.c_float(0), None) in (TC_ERR_TOO_LARGE, TC_ERR_ARG)
    # 250 x 250 outputs (62,500 rows) of 3 x 3 x 32 = 288 bytes: 18 MB > the 16 MiB buffer
    assert L.tc_conv_w8a8_noalloc(fake, 32, 250, 250, 32, 3, 3, 1, 1, fake, fake, 1, None, fake, 64, 16, 0, 0,
                                  ctypes.c_float(0), None) == TC_ERR_TOO_LARGE
    assert L.tc_conv_w8a8_noalloc(None, 32, 8, 8, 32, 3, 3, 1, 1, fake, fake, 1, None, fake, 64, 16, 0, 0,
                                  ctypes.c_float(0), None) == TC_ERR_ARG
    # padding as wide as the window, and an image of more than 2^31 pixels: refused before any work
    assert L.tc_conv_w8a8_noalloc(fake, 32, 8, 8, 32, 3, 3, 1, 3, fake, fake, 1, None, fake, 64, 16, 0, 0,
                                  ctypes.c_float(0), None) == TC_ERR_ARG
    assert L.tc_conv_w8a8_noalloc(fake, 32, 100000, 100000, 32, 3, 3, 1000, 1, fake, fake, 1, None, fake, 64, 16,
                                  0, 0, ctypes.c_float(0), None) == TC_ERR_ARG
