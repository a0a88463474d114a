#:set architecture = [('Conv', ['input'], [[1, 1], [3, 3], [1, 1, 1, 1], [1, 1]]), ('Relu', ['input'], [4]), ('MaxPool', ['input'], [0, [0, 0, 0, 0], [2, 2]]), ('Conv', ['input'], [[1, 1], [3, 3], [1, 1, 1, 1], [1, 1]]), ('Relu', ['input'], [4]), ('AveragePool', ['input'], [0, [0, 0, 0, 0], [2, 2]]), ('Reshape', ('input', 4), ['output0'], [[1, 54]], [0]), ('Gemm', ['output0', 1], None), ('Relu', ['output0'], [2]), ('Gemm', ['output0', 1], None)]
#:set inputs = [['output0', 2]]
#:set trueInputs = [['input', [1, 1, 12, 12]]]
#:set outShape = [['output', [1, 5]]]
#:set outputs = {'output': 'output0'}
