#:set architecture = [('Gemm', ['input', 1], None), ('Relu', ['input'], [2]), ('Gemm', ['input', 1], None), ('Relu', ['input'], [2]), ('Gemm', ['input', 1], None), ('Relu', ['input'], [2]), ('Gemm', ['input', 1], None), ('Relu', ['input'], [2]), ('Gemm', ['input', 1], None), ('Relu', ['input'], [2]), ('Gemm', ['input', 1], None)]
#:set inputs = []
#:set trueInputs = [['input', [1, 2]]]
#:set outShape = [['output', [1, 68]]]
#:set outputs = {'output': 'input'}
