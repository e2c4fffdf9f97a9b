"""Module path of the reference's FSDP2 bf16-NaN patch (models/gpt_oss/fsdp2_fix.py), imported
there for its side effect.  Nothing is patched here: torch canonicalises NaN bit patterns when
it copies bf16 tensors, which corrupted MXFP4 bytes stored in bf16 containers, but this package
keeps the MXFP4 blocks and scales in uint8 tensors end to end, so no copy can alter them."""
