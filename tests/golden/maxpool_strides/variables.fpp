#:set architecture = [('MaxPool', ['input'], [0, [0, 0, 0, 0], [1, 1]])]
#:set inputs = []
#:set trueInputs = [['input', [1, 2, 6, 6]]]
#:set outShape = [['output', [1, 2, 4, 4]]]
#:set outputs = {'output': 'input'}
