"""kvq: host side of the B200 4-bit KV-cache library (libkvq.so).

Put krea-realtime-bench_b200/ on sys.path; then `import quant_kv` and
`import quant_kv_kernels` give the drop-in modules, and `kvq` the lower-level
torch wrappers of the C ABI (kvq.ops), the library loader (kvq._lib), the build
recipe (kvq.build) and the synthetic workload generator (kvq.synth).
"""
