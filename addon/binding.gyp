{
  "targets": [{
    "target_name": "b2a",
    "sources": ["b2a_napi.c"],
    "include_dirs": ["../include"],
    "defines": ["B2A_HAVE_NODE_API_H"],
    "libraries": ["-L<(module_root_dir)/../llm-inference-webgpu_b200/b2a", "-lb2a",
                  "-Wl,-rpath,<(module_root_dir)/../llm-inference-webgpu_b200/b2a"]
  }]
}
