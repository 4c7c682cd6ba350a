{
  "targets": [
    {
      "target_name": "dllm_napi",
      "sources": ["dllm_napi.c"],
      "include_dirs": ["../../include"],
      "libraries": ["-L<(module_root_dir)/..", "-ldllm", "-Wl,-rpath,<(module_root_dir)/.."],
      "cflags": ["-O2", "-std=c11"]
    }
  ]
}
