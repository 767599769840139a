"""EXL3 trellis decode + matmul for B200 (sm_100a), behind the reference plugin's seams.

* :mod:`plugins_b200.quant` -- the quant seam (QuantTable: claims / validate / bill / open / load / matmul / swiglu)
  over ``libexl3b200.so`` (C ABI: ``include/exl3_b200.h``);
* :mod:`plugins_b200.model` -- the model seam narrowed to the EXL3 linears (claims, parse, bill, load, forward);
* :mod:`plugins_b200.pack` -- safetensors packs and config.json as the seams' tensor source;
* :mod:`plugins_b200.sharding` -- the splits over the GPUs of one box (column-parallel linears, expert-parallel and
  column-parallel experts);
* :mod:`plugins_b200.encoder` -- trellis encoding for synthetic weights;
* :mod:`plugins_b200.build` -- the in-tree sm_100a build; ``profile_gemv`` / ``profile_gemm`` / ``profile_moe`` --
  timing entry points (and ncu capture targets).
"""
