"""asap_b200: the A->F->A MoE round trip of the sgl-afd-plugin (ASAP) on B200.

Host side in Python over libasap.so (C ABI, include/asap.h), the sm_100a CUDA library that does the data path:
dispatch (route + pack + P2P stores + doorbell), the F rank's expert chain (doorbell wait, expert-major
permutation, MXFP8 quantisation, tcgen05 block-scaled GEMMs with fused SwiGLU / requantisation / top-k
weighting, reply), and the combine.

Reference API mirrored here:
  transport/          AttnChannel, FfnServer, Geometry, Job, Row, Ticket, errors  (transport/*.py)
  dispatcher.py       AsapDispatcher, AsapBuffer, AsapDispatchOutput   (srt/layers/moe/token_dispatcher/asap.py)
  layer.py            AsapMoE, get_moe_impl_class                     (srt/layers/moe/ep_moe/layer.py)
  scheduler.py        FfnScheduler.run_job / rows_of, JobTimer       (srt/managers/scheduler.py)
  args.py             the --asap-* flags and transport_geometry()     (srt/arg_groups/fields/asap.py,
                                                                        srt/server_args.py)
"""

__version__ = "0.1.0"
