#:set architecture = [('Gemm', ['input', 1], None), ('Gemm', ['input', 1], None)]
#:set inputs = []
#:set trueInputs = [['input', [1, 4]]]
#:set outShape = [['output', [1, 3]]]
#:set outputs = {'output': 'input'}
