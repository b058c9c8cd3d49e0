// A candidate with a type error: the worker must stop at the compile stage.
torch::Tensor kernel_fn(torch::Tensor x0) {
  int not_a_tensor = x0;
  return not_a_tensor;
}
