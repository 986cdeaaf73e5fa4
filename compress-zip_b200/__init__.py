"""compress_zip_b200: B200-native model-plus-coder path of compress-zip.

Package layout:
  csrc/          CUDA kernels (sm_100a) and the C-ABI host library libczg.so
  engine.py      ctypes binding of the C-ABI (include/czg.h) -- the GPU path
  container.py   CZIPv1 outer/inner header and chunk payload
  czm.py         .czm (safetensors) model file reader/writer
  tokenizer.py   BPE tokenizer over the model's embedded JSON
  outer_codec.py zstd-22 / brotli-11 outer layer (host)
  cli.py         compress/decompress drivers with the reference CLI's flags
  synth.py       seeded synthetic corpora and the random-init arch-2 model
"""
