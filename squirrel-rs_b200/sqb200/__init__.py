"""squirrel-b200: the B200 (sm_100a) implementation of squirrel-rs's Llama token
loop behind a C ABI (include/squirrel_cuda.h). `lib` binds the ABI; `gguf_synth`
writes the seeded random-init GGUF models the benches and parity tests use."""
